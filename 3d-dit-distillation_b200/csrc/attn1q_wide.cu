// The context->x attention of the exact 1-token branch without materialising the
// voxels' keys and values.  In the reference the single context query of each head
// attends over K = h Wk^T + bk and V = h Wv^T + bv, the rows of the cross linear of
// the modulated voxel stream h [n, D] (lib/fast_flow.py:1769-1777).  Since
//   q_h . K[r, h] = h[r] . (Wk_h^T q_h) + q_h . bk_h   (the second term is the same
//   for every key and cancels in the softmax), and
//   sum_r p[r, h] V[r, h] = Wv_h (sum_r p[r, h] h[r]) + bv_h   (sum_r p = 1),
// the attention runs on h directly: fold each query through Wk (qf [H, D] fp32),
// stream h once computing the H scores of every row in fp32 with an online softmax and
// the probability-weighted row sums u_h = sum_r p h[r] (split over row ranges), then
// combine the splits and apply Wv and bv.  HBM traffic: one read of h (n x D bf16)
// instead of writing and reading the [n, 2D] K/V.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace vdit {
namespace {

constexpr int kRows = 8;               // rows per batch of the streaming pass
constexpr int kHg = 4;                 // heads per block (kRows * kHg = 32 partial scores per thread)
constexpr int kMaxHeads = 16;
constexpr int kMinRowsPerRange = 64;   // shortest row range of the streaming pass
constexpr int kFoldThreads = 256;
constexpr int kCombThreads = 256;

// qf[h, d] = scale_log2 * sum_j q[h*hd + j] * wk[(h*hd + j), d]; a block covers 64 columns
// of one head, its four thread groups a quarter of the j range each
__global__ void __launch_bounds__(kFoldThreads) wide1q_fold_kernel(const __nv_bfloat16* __restrict__ q,
                                                                   const __nv_bfloat16* __restrict__ wk,
                                                                   int64_t ldw, int d, int hd, float scale_log2,
                                                                   float* __restrict__ qf) {
    __shared__ float qs[256];
    __shared__ float part[4][64];
    const int h = blockIdx.y;
    const int c = threadIdx.x & 63, jg = threadIdx.x >> 6;
    const int col = blockIdx.x * 64 + c;
    for (int j = threadIdx.x; j < hd; j += kFoldThreads) qs[j] = bf2f(q[(int64_t)h * hd + j]);
    __syncthreads();
    const int j0 = jg * hd / 4, j1 = (jg + 1) * hd / 4;
    float acc = 0.f;
    if (col < d) {
        const __nv_bfloat16* w = wk + (int64_t)h * hd * ldw + col;
#pragma unroll 8
        for (int j = j0; j < j1; ++j) acc = fmaf(qs[j], bf2f(w[(int64_t)j * ldw]), acc);
    }
    part[jg][c] = acc;
    __syncthreads();
    if (jg == 0 && col < d)
        qf[(int64_t)h * d + col] = ((part[0][c] + part[1][c]) + (part[2][c] + part[3][c])) * scale_log2;
}

// A block handles one range of rows for one group of kHg heads (the groups of a range
// are adjacent blocks, so the range's rows are read from HBM once and from L2 after).
// Thread t owns columns [4t, 4t + 4) of its heads' folded queries and weighted row sums.
// Per batch of kRows rows: kRows x kHg partial scores per thread, reduced across the warp
// by recursive halving (lane L ends with value L: row L / kHg, head L % kHg), then
// across warps through shared memory by warp 0, whose lanes (one per row and head) then
// update each head's running max / sum with shuffles and turn the scores into
// probabilities; every thread rescales and accumulates u.
__global__ void wide1q_partial_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t n, int d, int heads,
                                      const float* __restrict__ qf, int64_t per, float* __restrict__ ws) {
    constexpr int V = kRows * kHg;                   // 32: one reduced value per lane
    // double-buffered by batch parity, so a batch needs two barriers: one before warp 0 reduces
    // the warps' partial scores and runs the softmax, one before every thread reads the result
    __shared__ float red[2][16][V];                  // up to 512 threads
    __shared__ float sc[2][V];                       // probabilities
    __shared__ float alpha[2][kHg], mstate[kHg], lstate[kHg];
    const int ngroups = (heads + kHg - 1) / kHg;
    const int rr = blockIdx.x / ngroups, hg = blockIdx.x % ngroups;
    const int nwarps = blockDim.x >> 5;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int col = 4 * t;
    const int64_t r0 = (int64_t)rr * per, r1 = min(n, r0 + per);

    float q4[kHg][4], u[kHg][4];
#pragma unroll
    for (int hl = 0; hl < kHg; ++hl) {
        const int h = hg * kHg + hl;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            q4[hl][k] = h < heads ? qf[(int64_t)h * d + col + k] : 0.f;
            u[hl][k] = 0.f;
        }
    }
    // raw rows of the next batch are loaded while the current one is reduced
    uint2 nxt[kRows];
    auto fetch = [&](int64_t b) {
#pragma unroll
        for (int r = 0; r < kRows; ++r)
            nxt[r] = b + r < r1 ? __ldg(reinterpret_cast<const uint2*>(x + (b + r) * ldx + col)) : make_uint2(0u, 0u);
    };
    fetch(r0);
    float m_run = -INFINITY, l_run = 0.f;            // warp 0: the state of head lane % kHg
    int par = 0;
    for (int64_t b = r0; b < r1; b += kRows, par ^= 1) {
        float hv[kRows][4];
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&nxt[r]);
            const float2 a = __bfloat1622float2(p2[0]), c = __bfloat1622float2(p2[1]);
            hv[r][0] = a.x;
            hv[r][1] = a.y;
            hv[r][2] = c.x;
            hv[r][3] = c.y;
        }
        if (b + kRows < r1) fetch(b + kRows);
        float val[V];
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int hl = 0; hl < kHg; ++hl)
                val[r * kHg + hl] =
                    hv[r][0] * q4[hl][0] + hv[r][1] * q4[hl][1] + hv[r][2] * q4[hl][2] + hv[r][3] * q4[hl][3];
        // recursive halving across the warp: after step s a lane keeps the half picked by bit 4-s
#pragma unroll
        for (int s = 0; s < 5; ++s) {
            const int o = 16 >> s;
            const int half = V >> (s + 1);
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < half; ++i) {
                const float send = up ? val[i] : val[i + half];
                const float recv = __shfl_xor_sync(0xffffffffu, send, o);
                val[i] = (up ? val[i + half] : val[i]) + recv;
            }
        }
        red[par][warp][lane] = val[0];
        __syncthreads();
        if (warp == 0) {        // lane = row * kHg + head: online softmax of the batch, per head
            float sum = 0.f;
            for (int w = 0; w < nwarps; ++w) sum += red[par][w][lane];
            const int hl = lane % kHg;
            const float sv = (b + lane / kHg < r1) ? sum : -INFINITY;
            float mb = sv;
#pragma unroll
            for (int o = kHg; o < 32; o <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
            const float m_new = fmaxf(m_run, mb);
            const float a = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
            const float pr = exp2f(sv - m_new);
            float l = l_run * a;     // rows summed in order, as a serial loop would
#pragma unroll
            for (int r = 0; r < kRows; ++r) l += __shfl_sync(0xffffffffu, pr, r * kHg + hl);
            sc[par][lane] = pr;
            if (lane < kHg) alpha[par][lane] = a;
            m_run = m_new;
            l_run = l;
        }
        __syncthreads();
#pragma unroll
        for (int hl = 0; hl < kHg; ++hl) {
            const float a = alpha[par][hl];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float acc = u[hl][k] * a;
#pragma unroll
                for (int r = 0; r < kRows; ++r) acc = fmaf(sc[par][r * kHg + hl], hv[r][k], acc);
                u[hl][k] = acc;
            }
        }
    }
    if (warp == 0 && lane < kHg) {
        mstate[lane] = m_run;
        lstate[lane] = l_run;
    }
    __syncthreads();
    // partial state of this row range: per head [m, l, u[d]]
#pragma unroll
    for (int hl = 0; hl < kHg; ++hl) {
        const int h = hg * kHg + hl;
        if (h >= heads) break;
        float* o = ws + ((int64_t)rr * heads + h) * (d + 2);
        if (t == 0) {
            o[0] = mstate[hl];
            o[1] = lstate[hl];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) o[2 + col + k] = u[hl][k];
    }
}

// Merge the row ranges of one head (u / l at the common max) for 256 columns per block:
// ubar[h, c] = sum_s w_s u_s[c] / sum_s w_s l_s, w_s = 2^(m_s - max m).
__global__ void __launch_bounds__(kCombThreads) wide1q_merge_kernel(const float* __restrict__ ws, int splits,
                                                                    int heads, int d, float* __restrict__ ubar) {
    __shared__ float wsplit[1024];
    __shared__ float red[kCombThreads / 32];
    __shared__ float m_all, inv_l;
    const int h = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float m = -INFINITY;
    for (int s = t; s < splits; s += kCombThreads) m = fmaxf(m, ws[((int64_t)s * heads + h) * (d + 2)]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (t == 0) {
        float v = red[0];
        for (int w = 1; w < kCombThreads / 32; ++w) v = fmaxf(v, red[w]);
        m_all = v;
    }
    __syncthreads();
    float l = 0.f;
    for (int s = t; s < splits; s += kCombThreads) {
        const float* o = ws + ((int64_t)s * heads + h) * (d + 2);
        const float w = o[0] == -INFINITY ? 0.f : exp2f(o[0] - m_all);
        wsplit[s] = w;
        l += w * o[1];
    }
    l = warp_sum(l);
    __syncthreads();                 // red is reused
    if (lane == 0) red[warp] = l;
    __syncthreads();
    if (t == 0) {
        float v = 0.f;
        for (int w = 0; w < kCombThreads / 32; ++w) v += red[w];
        inv_l = 1.f / v;
    }
    __syncthreads();
    const int c = blockIdx.x * kCombThreads + t;
    if (c >= d) return;
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc = fmaf(wsplit[s], ws[((int64_t)s * heads + h) * (d + 2) + 2 + c], acc);
    ubar[(int64_t)h * d + c] = acc * inv_l;
}

// out[h*hd + j] = bf16(wv[h*hd + j, :] . ubar[h] + bv[h*hd + j]), one warp per output channel
__global__ void __launch_bounds__(kCombThreads) wide1q_project_kernel(const float* __restrict__ ubar, int heads, int d,
                                                                      int hd, const __nv_bfloat16* __restrict__ wv,
                                                                      int64_t ldw, const __nv_bfloat16* __restrict__ bv,
                                                                      __nv_bfloat16* __restrict__ out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t o = (int64_t)blockIdx.x * (kCombThreads / 32) + warp;     // output channel
    if (o >= (int64_t)heads * hd) return;
    const float* u = ubar + (o / hd) * d;
    const __nv_bfloat16* w = wv + o * ldw;
    float acc = 0.f;
    for (int c = lane * 8; c < d; c += 256) {
        float wf[8];
        load8_nc(w + c, wf);
        const float4 u0 = *reinterpret_cast<const float4*>(u + c);
        const float4 u1 = *reinterpret_cast<const float4*>(u + c + 4);
        acc = fmaf(wf[0], u0.x, acc);
        acc = fmaf(wf[1], u0.y, acc);
        acc = fmaf(wf[2], u0.z, acc);
        acc = fmaf(wf[3], u0.w, acc);
        acc = fmaf(wf[4], u1.x, acc);
        acc = fmaf(wf[5], u1.y, acc);
        acc = fmaf(wf[6], u1.z, acc);
        acc = fmaf(wf[7], u1.w, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) out[o] = f2bf(acc + bf2f(bv[o]));
}

// Row ranges of the streaming pass: one wave of CTAs (ranges x head groups = the SM count, one
// CTA per SM) unless the ranges would get shorter than kMinRowsPerRange rows.  At n = 16384,
// 12 heads: 49 ranges of 335 rows, 147 CTAs, against 128 ranges of 128 rows in 2.6 waves, which
// measured 7% slower (and 64 ranges of 256 rows in 1.3 waves 17% slower).  The merge kernel takes
// at most 1024 ranges.
int splits_for(int64_t n, int heads) {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            sms = 148;
    }
    const int ngroups = std::max(1, (heads + kHg - 1) / kHg);
    const int64_t wave = std::max(1, sms / ngroups);
    const int64_t most = (n + kMinRowsPerRange - 1) / kMinRowsPerRange;
    return (int)std::max<int64_t>(1, std::min<int64_t>(1024, std::min(wave, most)));
}

}  // namespace
}  // namespace vdit

using namespace vdit;

extern "C" size_t vdit_attention_1q_wide_workspace_bytes(int32_t heads, int32_t head_dim, int64_t n_keys) {
    const int64_t d = (int64_t)heads * head_dim;
    return (size_t)heads * (size_t)(d + 2) * sizeof(float) * (size_t)(2 + splits_for(n_keys, heads));
}

extern "C" int vdit_attention_1q_wide(const void* q, const void* x, int64_t ldx, int64_t n, const void* wk,
                                      const void* wv, int64_t ldw, const void* bv, int32_t heads, int32_t head_dim,
                                      float softmax_scale, void* out, void* workspace, size_t workspace_bytes,
                                      vdit_stream_t stream) {
    if (!q || !x || !wk || !wv || !bv || !out || !workspace || n < 1 || heads < 1 || head_dim < 1) return VDIT_ERR_ARG;
    const int64_t d = (int64_t)heads * head_dim;
    if (heads > kMaxHeads || d % 128 || d > 2048 || head_dim > 256) return VDIT_ERR_UNSUPPORTED;
    if (ldx < d || ldw < d) return VDIT_ERR_ARG;
    if (!aligned16(x) || !aligned16(wv) || !aligned16(workspace) || ldx % 8 || ldw % 8) return VDIT_ERR_ALIGN;
    if (workspace_bytes < vdit_attention_1q_wide_workspace_bytes(heads, head_dim, n)) return VDIT_ERR_WORKSPACE;
    const int splits = splits_for(n, heads);
    float* qf = static_cast<float*>(workspace);  // heads x d, then ubar heads x d, then splits x heads x (d + 2)
    float* ubar = qf + heads * d;
    float* ws = ubar + heads * d;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float scale_log2 = softmax_scale * 1.4426950408889634f;
    wide1q_fold_kernel<<<dim3((unsigned)((d + 63) / 64), heads), kFoldThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(wk), ldw, (int)d, head_dim,
        scale_log2, qf);
    const int threads = (int)(d / 4);            // 32..512
    const int64_t per = (n + splits - 1) / splits;
    const int ngroups = (heads + kHg - 1) / kHg;
    wide1q_partial_kernel<<<(unsigned)(splits * ngroups), threads, 0, s>>>(static_cast<const __nv_bfloat16*>(x), ldx,
                                                                            n, (int)d, heads, qf, per, ws);
    wide1q_merge_kernel<<<dim3((unsigned)((d + kCombThreads - 1) / kCombThreads), heads), kCombThreads, 0, s>>>(
        ws, splits, heads, (int)d, ubar);
    wide1q_project_kernel<<<(unsigned)((heads * head_dim + kCombThreads / 32 - 1) / (kCombThreads / 32)),
                            kCombThreads, 0, s>>>(ubar, heads, (int)d, head_dim,
                                                  static_cast<const __nv_bfloat16*>(wv), ldw,
                                                  static_cast<const __nv_bfloat16*>(bv),
                                                  static_cast<__nv_bfloat16*>(out));
    count_launches(4);
    return check_launch();
}
