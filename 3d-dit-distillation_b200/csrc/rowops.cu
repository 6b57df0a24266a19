// Row-wise fused kernels of the DiT block: AdaLN modulation, gate-add,
// QK-RMSNorm + RoPE (+ Hilbert gather), packed SwiGLU, patchify, output
// modulation + unpatchify, and the small sampler kernels.  All are HBM-bound:
// rows move through registers/shared memory in 16-byte vectors, statistics
// are reduced with warp shuffles in fp32.
#include "common.cuh"

namespace vdit {
namespace {

constexpr int kRowWarps = 8;            // rows per 256-thread block
constexpr int kMaxVec = 8;              // 16-byte vectors per lane -> d <= 2048

// ---------------------------------------------------------------- LN helpers
// One warp per row; lane l holds vectors l, l+32, ... of the row (8 values each).
struct RowRegs {
    float v[kMaxVec][8];
};

__device__ __forceinline__ void row_load(const __nv_bfloat16* __restrict__ row, int nvec, int lane, RowRegs& r) {
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        int vi = lane + 32 * i;
        if (vi < nvec) load8(row + vi * 8, r.v[i]);
    }
}

__device__ __forceinline__ void row_stats(const RowRegs& r, int nvec, int lane, int d, float& mean, float& rstd) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i)
        if (lane + 32 * i < nvec)
#pragma unroll
            for (int j = 0; j < 8; ++j) s += r.v[i][j];
    mean = warp_sum(s) / (float)d;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i)
        if (lane + 32 * i < nvec)
#pragma unroll
            for (int j = 0; j < 8; ++j) { float t = r.v[i][j] - mean; q += t * t; }
    rstd = rsqrtf(warp_sum(q) / (float)d + 1e-6f);
}

__device__ __forceinline__ void row_modulate_store(const RowRegs& r, int nvec, int lane, float mean, float rstd,
                                                   const float* __restrict__ s1, const float* __restrict__ sh,
                                                   __nv_bfloat16* __restrict__ out) {
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        int vi = lane + 32 * i;
        if (vi >= nvec) continue;
        float4 a0 = __ldg(reinterpret_cast<const float4*>(s1 + vi * 8));
        float4 a1 = __ldg(reinterpret_cast<const float4*>(s1 + vi * 8 + 4));
        float4 b0 = __ldg(reinterpret_cast<const float4*>(sh + vi * 8));
        float4 b1 = __ldg(reinterpret_cast<const float4*>(sh + vi * 8 + 4));
        float sa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        float sb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (r.v[i][j] - mean) * rstd * sa[j] + sb[j];
        store8(out + vi * 8, o);
    }
}

__global__ void __launch_bounds__(256) modulate_kernel(const __nv_bfloat16* __restrict__ x, int64_t m, int d,
                                                       const float* __restrict__ s1, const float* __restrict__ sh,
                                                       __nv_bfloat16* __restrict__ out) {
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t row = blockIdx.x * (int64_t)kRowWarps + warp;
    if (row >= m) return;
    int nvec = d >> 3;
    RowRegs r;
    row_load(x + row * d, nvec, lane, r);
    float mean, rstd;
    row_stats(r, nvec, lane, d, mean, rstd);
    row_modulate_store(r, nvec, lane, mean, rstd, s1, sh, out + row * d);
}

// x <- bf16(x + h * g); optional mod_out = LN(x) * s1 + sh
__global__ void __launch_bounds__(256) gate_add_modulate_kernel(
    __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ h, int64_t h_stride, int64_t m, int d,
    const float* __restrict__ g, const float* __restrict__ s1, const float* __restrict__ sh,
    __nv_bfloat16* __restrict__ mod_out) {
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t row = blockIdx.x * (int64_t)kRowWarps + warp;
    if (row >= m) return;
    int nvec = d >> 3;
    RowRegs r;
    __nv_bfloat16* xr = x + row * d;
    const __nv_bfloat16* hr = h + row * h_stride;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        int vi = lane + 32 * i;
        if (vi >= nvec) continue;
        float xv[8], hv[8];
        load8(xr + vi * 8, xv);
        load8(hr + vi * 8, hv);
        float4 g0 = __ldg(reinterpret_cast<const float4*>(g + vi * 8));
        float4 g1 = __ldg(reinterpret_cast<const float4*>(g + vi * 8 + 4));
        float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        uint4 packed;
        __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            p2[j] = __floats2bfloat162_rn(xv[2 * j] + hv[2 * j] * gg[2 * j], xv[2 * j + 1] + hv[2 * j + 1] * gg[2 * j + 1]);
            float2 t = __bfloat1622float2(p2[j]);
            r.v[i][2 * j] = t.x;
            r.v[i][2 * j + 1] = t.y;
        }
        *reinterpret_cast<uint4*>(xr + vi * 8) = packed;
    }
    if (mod_out == nullptr) return;
    float mean, rstd;
    row_stats(r, nvec, lane, d, mean, rstd);
    row_modulate_store(r, nvec, lane, mean, rstd, s1, sh, mod_out + row * d);
}

// out[row, o] = sum_c bf16(LN(x)*s1+sh)[c] * w[o, c], 16 outputs, fp32
__global__ void __launch_bounds__(256) out_unpatchify_kernel(const __nv_bfloat16* __restrict__ x, int64_t m, int d,
                                                             const float* __restrict__ s1, const float* __restrict__ sh,
                                                             const float* __restrict__ w, float* __restrict__ out) {
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t row = blockIdx.x * (int64_t)kRowWarps + warp;
    if (row >= m) return;
    int nvec = d >> 3;
    RowRegs r;
    row_load(x + row * d, nvec, lane, r);
    float mean, rstd;
    row_stats(r, nvec, lane, d, mean, rstd);
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        int vi = lane + 32 * i;
        if (vi >= nvec) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float y = (r.v[i][j] - mean) * rstd * __ldg(s1 + vi * 8 + j) + __ldg(sh + vi * 8 + j);
            r.v[i][j] = bf2f(f2bf(y));
        }
    }
    float acc[16];
#pragma unroll
    for (int o = 0; o < 16; ++o) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxVec; ++i) {
            int vi = lane + 32 * i;
            if (vi >= nvec) continue;
            const float4* wp = reinterpret_cast<const float4*>(w + (int64_t)o * d + vi * 8);
            float4 w0 = __ldg(wp), w1 = __ldg(wp + 1);
            s += r.v[i][0] * w0.x + r.v[i][1] * w0.y + r.v[i][2] * w0.z + r.v[i][3] * w0.w +
                 r.v[i][4] * w1.x + r.v[i][5] * w1.y + r.v[i][6] * w1.z + r.v[i][7] * w1.w;
        }
        acc[o] = warp_sum(s);
    }
    if (lane < 16) {
        float v = acc[0];
#pragma unroll
        for (int o = 1; o < 16; ++o) if (lane == o) v = acc[o];
        out[row * 16 + lane] = v;
    }
}

// ---------------------------------------------------------------- QK norm + RoPE
// One warp per token row, looping over its heads: lanes 0..15 hold a head's q
// vector, lanes 16..31 its k vector (8 channels each, one 16-byte load per lane;
// head_dim 96 uses 12 lanes per half).  The token's source index, coordinates
// and the RoPE cos/sin of each lane's 8 channels are fetched once and reused
// for every head; the next head's vectors are loaded while the current one is
// normalised.  RMS statistics reduce over the 16-lane half with shuffles; the
// normalised values go through a per-warp shared-memory slot so each lane can
// read its RoPE partner channel (e +- M); v is copied through.
//   MODE 0: 3D RoPE, positions from h_coords[src] via the [res, hd/6] tables,
//           optional gather src = fwd[dst].
//   MODE 1: 2D RoPE on tokens >= n_prefix via [L-n_prefix, 2, hd/4] tables, in place.
constexpr int kQkWarps = 8;

template <int MODE>
__global__ void __launch_bounds__(kQkWarps * 32) qknorm_rope_kernel(
    const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int64_t rows, int heads, int hd,
    const float* __restrict__ qs, const float* __restrict__ ks, const float* __restrict__ cs,
    const float* __restrict__ sn, int res, const int4* __restrict__ hc, const int64_t* __restrict__ fwd,
    int n_prefix) {
    __shared__ float snorm[kQkWarps][2][128];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t dst = (int64_t)blockIdx.x * kQkWarps + warp;
    if (dst >= rows) return;
    const int64_t src = (MODE == 0 && fwd != nullptr) ? fwd[dst] : dst;
    const int D = heads * hd;
    const int half = lane >> 4, vi = lane & 15;                 // half 0 = q, 1 = k
    const bool active = vi * 8 < hd;
    const __nv_bfloat16* irow = in + src * (int64_t)(3 * D);
    __nv_bfloat16* orow = out + dst * (int64_t)(3 * D);

    // RoPE of this lane's 8 channels (identical for every head)
    const int naxes = MODE == 0 ? 3 : 2;
    const int M = hd / (2 * naxes);
    bool rotate = true;
    int64_t tab_row[3] = {0, 0, 0};
    if (MODE == 0) {
        const int4 c = hc[src];
        tab_row[0] = min(max(c.y, 0), res - 1);
        tab_row[1] = min(max(c.z, 0), res - 1);
        tab_row[2] = min(max(c.w, 0), res - 1);
    } else {
        rotate = dst >= n_prefix;
        const int64_t pt = dst - n_prefix;
        tab_row[0] = pt * 2;
        tab_row[1] = pt * 2 + 1;
    }
    float rc[8], rs[8];
    int partner[8];            // channel index of the RoPE partner, -1: channel passes through
    bool lower[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int e = vi * 8 + j;
        const int grp = e / (2 * M), off = e - grp * 2 * M;
        rc[j] = 1.f;
        rs[j] = 0.f;
        partner[j] = -1;
        lower[j] = true;
        if (active && rotate && grp < naxes) {
            const int f = off < M ? off : off - M;
            rc[j] = __ldg(cs + tab_row[grp] * M + f);
            rs[j] = __ldg(sn + tab_row[grp] * M + f);
            lower[j] = off < M;
            partner[j] = lower[j] ? e + M : e - M;
        }
    }

    float* nb = snorm[warp][half];
    float x[8] = {0, 0, 0, 0, 0, 0, 0, 0};        // lanes past head_dim must add zeros to the RMS sum
    uint4 vcopy = make_uint4(0, 0, 0, 0);
    if (active) {
        load8(irow + half * D + vi * 8, x);
        if (half == 0) vcopy = *reinterpret_cast<const uint4*>(irow + 2 * D + vi * 8);
    }
    for (int h = 0; h < heads; ++h) {
        // prefetch the next head's vectors
        float xn[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        uint4 vn = make_uint4(0, 0, 0, 0);
        if (active && h + 1 < heads) {
            load8(irow + half * D + (h + 1) * hd + vi * 8, xn);
            if (half == 0) vn = *reinterpret_cast<const uint4*>(irow + 2 * D + (h + 1) * hd + vi * 8);
        }
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rr = rsqrtf(ss / (float)hd + 1e-6f);
        const float* scale = (half == 0 ? qs : ks) + h * hd;
        __syncwarp();                                    // the previous head's partner reads are done
        if (active) {
            const float4 s0 = __ldg(reinterpret_cast<const float4*>(scale + vi * 8));
            const float4 s1 = __ldg(reinterpret_cast<const float4*>(scale + vi * 8 + 4));
            const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                x[j] = bf2f(f2bf(x[j] * rr)) * sc[j];        // normalised value rounded like the reference
                nb[vi * 8 + j] = x[j];
            }
        }
        __syncwarp();
        if (active) {
            float o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                o[j] = x[j];
                if (partner[j] >= 0) {
                    const float pv = nb[partner[j]];
                    o[j] = lower[j] ? x[j] * rc[j] - pv * rs[j] : x[j] * rc[j] + pv * rs[j];
                }
            }
            store8(orow + half * D + h * hd + vi * 8, o);
            if (half == 0) *reinterpret_cast<uint4*>(orow + 2 * D + h * hd + vi * 8) = vcopy;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = xn[j];
        vcopy = vn;
    }
}

// ---------------------------------------------------------------- misc
__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ h, int64_t m, int f, __nv_bfloat16* __restrict__ out) {
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int fv = f >> 3;
    if (t >= m * fv) return;
    int64_t row = t / fv;
    int c = (int)(t % fv) * 8;
    float a[8], g[8], o[8];
    load8(h + row * 2 * f + c, a);
    load8(h + row * 2 * f + f + c, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = silu(g[j]) * a[j];
    store8(out + row * f + c, o);
}

// x[n, d] = xt[n,16] @ w[d,16]^T.  A block owns 64 output channels for many rows:
// their 64x16 weights sit in registers (lane = one output channel pair), each
// warp streams rows, reading a row's 16 inputs once (broadcast) and writing
// 64 outputs per row.
constexpr int kPatchRows = 64;

__global__ void __launch_bounds__(256) patchify_kernel(const float* __restrict__ xt, int64_t n,
                                                       const float* __restrict__ w, int d,
                                                       __nv_bfloat16* __restrict__ out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = blockIdx.x * 64 + lane * 2;             // this lane's two output channels
    if (c0 >= d) return;
    float wa[16], wb[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        wa[i] = __ldg(w + (int64_t)c0 * 16 + i);
        wb[i] = __ldg(w + (int64_t)(c0 + 1) * 16 + i);
    }
    const int64_t r0 = (int64_t)blockIdx.y * kPatchRows;
    for (int64_t r = r0 + warp; r < min(n, r0 + kPatchRows); r += 8) {
        const float4* xp = reinterpret_cast<const float4*>(xt + r * 16);
        float x[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 q = __ldg(xp + i);
            x[4 * i] = q.x; x[4 * i + 1] = q.y; x[4 * i + 2] = q.z; x[4 * i + 3] = q.w;
        }
        float sa = 0.f, sb = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            sa = fmaf(x[i], wa[i], sa);
            sb = fmaf(x[i], wb[i], sb);
        }
        *reinterpret_cast<__nv_bfloat162*>(out + r * d + c0) = __floats2bfloat162_rn(sa, sb);
    }
}

__global__ void gather_rows_f32_kernel(const float* __restrict__ src, const int64_t* __restrict__ idx, int64_t n, int c,
                                       float* __restrict__ dst) {
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (t >= n * c) return;
    int64_t r = t / c;
    dst[t] = src[idx[r] * c + (t % c)];
}

__global__ void cfg_euler_kernel(float* __restrict__ xt, const float* __restrict__ vp, const float* __restrict__ vn,
                                 int64_t total, float g, float dt) {
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (t >= total) return;
    float v = vp[t];
    if (vn) v = v + g * (v - vn[t]);
    xt[t] = xt[t] - dt * v;
}

__global__ void unpermute_denorm_kernel(const float* __restrict__ xt, const int64_t* __restrict__ up, int64_t n,
                                        const float* __restrict__ sc, const float* __restrict__ shf, float* __restrict__ out) {
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (t >= n * 16) return;
    int64_t i = t >> 4;
    int c = (int)(t & 15);
    out[t] = xt[up[i] * 16 + c] * sc[c] + shf[c];
}

inline unsigned blocks_for(int64_t n, int per) { return (unsigned)((n + per - 1) / per); }

}  // namespace
}  // namespace vdit

using namespace vdit;

static bool row_width_ok(int32_t d) { return d > 0 && d % 8 == 0 && d <= 256 * kMaxVec; }

extern "C" int vdit_patchify(const float* xt, int64_t n, const float* w, int32_t d, void* x_out, vdit_stream_t stream) {
    if (n < 0 || d <= 0 || d % 8 || !xt || !w || !x_out) return VDIT_ERR_ARG;
    if (!aligned16(xt) || !aligned16(w) || !aligned16(x_out)) return VDIT_ERR_ALIGN;
    if (n == 0) return VDIT_OK;
    if (d % 2) return VDIT_ERR_UNSUPPORTED;
    patchify_kernel<<<dim3((d + 63) / 64, (unsigned)((n + kPatchRows - 1) / kPatchRows)), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(xt, n, w, d, static_cast<__nv_bfloat16*>(x_out));
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_modulate(const void* x, int64_t m, int32_t d, const float* s1, const float* sh, void* out,
                             vdit_stream_t stream) {
    if (m < 0 || !row_width_ok(d) || !x || !s1 || !sh || !out) return VDIT_ERR_ARG;
    if (!aligned16(x) || !aligned16(out) || !aligned16(s1) || !aligned16(sh)) return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    modulate_kernel<<<blocks_for(m, kRowWarps), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(x), m, d, s1, sh, static_cast<__nv_bfloat16*>(out));
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_gate_add_modulate(void* x, const void* h, int64_t h_stride, int64_t m, int32_t d, const float* g,
                                      const float* s1, const float* sh, void* mod_out, vdit_stream_t stream) {
    if (m < 0 || !row_width_ok(d) || !x || !h || !g || h_stride < 0) return VDIT_ERR_ARG;
    if (mod_out && (!s1 || !sh)) return VDIT_ERR_ARG;
    if (!aligned16(x) || !aligned16(h) || !aligned16(g) || (h_stride % 8) || (mod_out && !aligned16(mod_out)) ||
        (s1 && !aligned16(s1)) || (sh && !aligned16(sh)))
        return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    gate_add_modulate_kernel<<<blocks_for(m, kRowWarps), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(h), h_stride, m, d, g, s1, sh,
        static_cast<__nv_bfloat16*>(mod_out));
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_out_modulate_unpatchify(const void* x, int64_t m, int32_t d, const float* s1, const float* sh,
                                            const float* w, float* out, vdit_stream_t stream) {
    if (m < 0 || !row_width_ok(d) || !x || !s1 || !sh || !w || !out) return VDIT_ERR_ARG;
    if (!aligned16(x) || !aligned16(w) || !aligned16(s1) || !aligned16(sh)) return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    out_unpatchify_kernel<<<blocks_for(m, kRowWarps), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(x), m, d, s1, sh, w, out);
    count_launches(1);
    return check_launch();
}


extern "C" int vdit_qknorm_rope3d_gather(const void* qkv, int64_t n, int32_t heads, int32_t hd, const float* qs,
                                         const float* ks, const float* cs, const float* sn, int32_t res,
                                         const int32_t* h_coords, const int64_t* fwd, void* out, vdit_stream_t stream) {
    if (n < 0 || heads < 1 || hd < 6 || hd % 8 || !qkv || !qs || !ks || !cs || !sn || !h_coords || !out || res < 1)
        return VDIT_ERR_ARG;
    if (qkv == out && fwd != nullptr) return VDIT_ERR_ARG;     // a gather cannot run in place
    if (!aligned16(qkv) || !aligned16(out) || !aligned16(h_coords)) return VDIT_ERR_ALIGN;
    if (n == 0) return VDIT_OK;
    if (hd > 128) return VDIT_ERR_UNSUPPORTED;
    qknorm_rope_kernel<0><<<blocks_for(n, kQkWarps), kQkWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(out), n, heads, hd, qs, ks, cs, sn, res,
        reinterpret_cast<const int4*>(h_coords), fwd, 0);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_qknorm_rope2d(void* qkv, int64_t l, int32_t heads, int32_t hd, const float* qs, const float* ks,
                                  const float* cs, const float* sn, int32_t n_prefix, vdit_stream_t stream) {
    if (l < 0 || heads < 1 || hd < 4 || hd % 8 || !qkv || !qs || !ks || n_prefix < 0) return VDIT_ERR_ARG;
    if (l > n_prefix && (!cs || !sn)) return VDIT_ERR_ARG;
    if (!aligned16(qkv)) return VDIT_ERR_ALIGN;
    if (l == 0) return VDIT_OK;
    if (hd > 128) return VDIT_ERR_UNSUPPORTED;
    qknorm_rope_kernel<1><<<blocks_for(l, kQkWarps), kQkWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(qkv), l, heads, hd, qs, ks, cs, sn, 1,
        nullptr, nullptr, n_prefix);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_swiglu_packed(const void* h, int64_t m, int32_t f, void* out, vdit_stream_t stream) {
    if (m < 0 || f <= 0 || f % 8 || !h || !out) return VDIT_ERR_ARG;
    if (!aligned16(h) || !aligned16(out)) return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    swiglu_kernel<<<blocks_for(m * (f / 8), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(h), m, f, static_cast<__nv_bfloat16*>(out));
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_gather_rows_f32(const float* src, const int64_t* idx, int64_t n, int32_t c, float* dst,
                                    vdit_stream_t stream) {
    if (n < 0 || c <= 0 || !src || !idx || !dst) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    gather_rows_f32_kernel<<<blocks_for(n * c, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(src, idx, n, c, dst);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_cfg_euler(float* xt, const float* vp, const float* vn, int64_t n, float g, float dt,
                              vdit_stream_t stream) {
    if (n < 0 || !xt || !vp) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    cfg_euler_kernel<<<blocks_for(n * 16, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(xt, vp, vn, n * 16, g, dt);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_unpermute_denorm(const float* xt, const int64_t* up, int64_t n, const float* sc, const float* shf,
                                     float* out, vdit_stream_t stream) {
    if (n < 0 || !xt || !up || !sc || !shf || !out) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    unpermute_denorm_kernel<<<blocks_for(n * 16, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(xt, up, n, sc, shf, out);
    count_launches(1);
    return check_launch();
}
