// Matrix-vector products for the one-row linears of the path: the context vector of the
// exact 1-token unconditional branch and the time-embedding / gate MLP.
//
//   out[b][r] = act( sum_i W[b][r][i] * x'[b][i] + bias[b][r] ),   r < n, i < k, b < batch
//
// x' is the input vector after an optional fused prologue (kept in shared memory as fp32):
//   VDIT_GEMV_X_BF16    x' = x (bf16 [k])
//   VDIT_GEMV_X_F32     x' = x (fp32 [k])
//   VDIT_GEMV_X_LN_MOD  x' = bf16(LN(x) * s1 + sh), x fp32 [k], LayerNorm without affine,
//                       eps 1e-6, two-pass fp32 statistics (the modulated context vector)
//   VDIT_GEMV_X_SWIGLU  x' = bf16(silu(g) * a) with x bf16 [2k] = [a | g] (the packed FFN hidden)
// W is bf16 or fp32 [n, k] per batch entry (bias of the same type, or none); accumulation is
// fp32; out is bf16 or fp32, with an optional silu.
//
// The products are HBM-bound (each weight byte is read once): every warp streams whole
// weight rows with 16-byte loads, four chunks of the row in flight per lane, and reduces
// the row with shuffles.  A CTA of 8 warps takes 8 consecutive rows per step; CTAs stride
// over the rows of their batch entry.
#include <algorithm>

#include "common.cuh"

namespace vdit {
namespace gemv {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int kMaxK = 8192;       // x' in shared memory: 32 KB of fp32 (no opt-in needed)

struct Args {
    int x_mode;
    const void* x;
    int64_t x_bstride;            // elements between batch entries (0: one vector for all)
    const float* s1;
    const float* sh;
    int64_t mod_bstride;
    const void* w;
    int64_t w_bstride;
    const void* bias;
    int64_t bias_bstride;
    void* out;
    int64_t out_bstride;
    int n, k, out_f32, silu_out;
};

__device__ __forceinline__ float block_sum(float t, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    t = warp_sum(t);
    __syncthreads();
    if (lane == 0) red[warp] = t;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) r += red[w];
    return r;
}

// 16 bytes of a weight row as fp32: 8 bf16 or 4 fp32 values
template <typename WT>
struct Chunk;
template <>
struct Chunk<__nv_bfloat16> {
    static constexpr int E = 8;
    __device__ __forceinline__ static void to_f32(const uint4& u, float* f) { unpack8(u, f); }
};
template <>
struct Chunk<float> {
    static constexpr int E = 4;
    __device__ __forceinline__ static void to_f32(const uint4& u, float* f) {
        f[0] = __uint_as_float(u.x);
        f[1] = __uint_as_float(u.y);
        f[2] = __uint_as_float(u.z);
        f[3] = __uint_as_float(u.w);
    }
};

template <typename WT>
__global__ void __launch_bounds__(THREADS) gemv_kernel(const __grid_constant__ Args a) {
    extern __shared__ float xs[];
    __shared__ float red[WARPS];
    const int b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = a.k;

    // ---------------------------------------------------------------- prologue: x' into shared memory
    if (a.x_mode == VDIT_GEMV_X_BF16) {
        const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(a.x) + b * a.x_bstride;
        for (int i = tid; i < k; i += THREADS) xs[i] = bf2f(x[i]);
    } else if (a.x_mode == VDIT_GEMV_X_F32) {
        const float* x = static_cast<const float*>(a.x) + b * a.x_bstride;
        for (int i = tid; i < k; i += THREADS) xs[i] = x[i];
    } else if (a.x_mode == VDIT_GEMV_X_LN_MOD) {
        const float* x = static_cast<const float*>(a.x) + b * a.x_bstride;
        const float* s1 = a.s1 + b * a.mod_bstride;
        const float* sh = a.sh + b * a.mod_bstride;
        float s = 0.f;
        for (int i = tid; i < k; i += THREADS) {
            const float v = x[i];
            xs[i] = v;
            s += v;
        }
        const float mean = block_sum(s, red) / (float)k;
        float q = 0.f;
        for (int i = tid; i < k; i += THREADS) q += (xs[i] - mean) * (xs[i] - mean);
        const float rstd = rsqrtf(block_sum(q, red) / (float)k + 1e-6f);
        for (int i = tid; i < k; i += THREADS) xs[i] = bf2f(f2bf((xs[i] - mean) * rstd * s1[i] + sh[i]));
    } else {   // VDIT_GEMV_X_SWIGLU
        const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(a.x) + b * a.x_bstride;
        for (int i = tid; i < k; i += THREADS) xs[i] = bf2f(f2bf(silu(bf2f(x[k + i])) * bf2f(x[i])));
    }
    __syncthreads();

    // ---------------------------------------------------------------- rows
    using C = Chunk<WT>;
    constexpr int E = C::E;
    const WT* wb = static_cast<const WT*>(a.w) + b * a.w_bstride;
    const WT* bias = a.bias ? static_cast<const WT*>(a.bias) + b * a.bias_bstride : nullptr;
    const int nchunks = k / E;                      // 16-byte chunks per row
    for (int r0 = blockIdx.x * WARPS; r0 < a.n; r0 += gridDim.x * WARPS) {
        const int r = r0 + warp;
        if (r >= a.n) break;
        const uint4* wr = reinterpret_cast<const uint4*>(wb + (int64_t)r * k);
        float acc = 0.f;
        int c = lane;
        for (; c + 96 < nchunks; c += 128) {       // four chunks in flight per lane
            uint4 u[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) u[j] = __ldg(wr + c + 32 * j);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float f[E];
                C::to_f32(u[j], f);
                const float* xv = xs + (c + 32 * j) * E;
#pragma unroll
                for (int e = 0; e < E; ++e) acc = fmaf(f[e], xv[e], acc);
            }
        }
        for (; c < nchunks; c += 32) {
            float f[E];
            C::to_f32(__ldg(wr + c), f);
            const float* xv = xs + c * E;
#pragma unroll
            for (int e = 0; e < E; ++e) acc = fmaf(f[e], xv[e], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) {
            if (bias) acc += (float)bias[r];
            if (a.silu_out) acc = silu(acc);
            if (a.out_f32)
                static_cast<float*>(a.out)[b * a.out_bstride + r] = acc;
            else
                static_cast<__nv_bfloat16*>(a.out)[b * a.out_bstride + r] = f2bf(acc);
        }
    }
}

int num_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        n = 148;
    return n;
}

}  // namespace gemv
}  // namespace vdit

using namespace vdit;

extern "C" int vdit_gemv(int32_t x_mode, const void* x, int64_t x_bstride, const float* mod_scale,
                         const float* mod_shift, int64_t mod_bstride, int32_t w_f32, const void* w, int64_t w_bstride,
                         const void* bias, int64_t bias_bstride, int32_t out_f32, int32_t silu_out, void* out,
                         int64_t out_bstride, int32_t n, int32_t k, int32_t batch, vdit_stream_t stream) {
    using namespace vdit::gemv;
    if (!x || !w || !out || n <= 0 || k <= 0 || batch <= 0 || x_bstride < 0 || w_bstride < 0 || bias_bstride < 0 ||
        out_bstride < 0 || mod_bstride < 0)
        return VDIT_ERR_ARG;
    if (x_mode < VDIT_GEMV_X_BF16 || x_mode > VDIT_GEMV_X_SWIGLU) return VDIT_ERR_ARG;
    if (x_mode == VDIT_GEMV_X_LN_MOD && (!mod_scale || !mod_shift)) return VDIT_ERR_ARG;
    if (k > kMaxK) return VDIT_ERR_UNSUPPORTED;
    const int e = w_f32 ? 4 : 8;                  // weight elements per 16-byte chunk
    if (k % e || (batch > 1 && w_bstride % e)) return VDIT_ERR_ALIGN;
    if (!aligned16(w)) return VDIT_ERR_ALIGN;
    if (batch > 1 && (w_bstride < (int64_t)n * k || out_bstride < n)) return VDIT_ERR_ARG;
    Args a{x_mode, x, x_bstride, mod_scale, mod_shift, mod_bstride, w, w_bstride, bias, bias_bstride, out,
           out_bstride, n, k, out_f32 != 0, silu_out != 0};
    const int ctas = std::min((n + WARPS - 1) / WARPS, num_sms() * 8);
    const dim3 grid(ctas, batch);
    const size_t smem = (size_t)k * sizeof(float);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (w_f32)
        gemv_kernel<float><<<grid, THREADS, smem, s>>>(a);
    else
        gemv_kernel<__nv_bfloat16><<<grid, THREADS, smem, s>>>(a);
    count_launches(1);
    return check_launch();
}
