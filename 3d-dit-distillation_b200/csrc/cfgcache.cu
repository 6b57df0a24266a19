// Approximate CFG cache of the sampler (opt-in, not part of the exact solver): on a guided
// step that skips the unconditional NFE, the last unconditional velocity is reused
// (the reference's cfg_cache_mode "neg_reuse", lib/fast_flow.py:2791-2887, non-QAOA branch):
//
//   nc    = last_neg, or (1 - a) * last_neg + a * (xt - x0) / t   (clean-endpoint blend;
//           x0 = xt_eval - t_eval * v_neg at the step that evaluated it, a = 0 disables it)
//   s     = clamp(sum(vp * nc) / max(sum(nc * nc), 1e-6), 0.9, 1.1)     (CFG-Zero* projection)
//   delta = vp - s * nc;   delta += hf * (delta - mean_rows(delta))      (high-frequency boost)
//   xt   -= dt * (vp + g * delta)
//
// (with the projection off: delta = vp - last_neg, no blend, no boost).  Latents are [n, 16]
// fp32.  Two launches with a fixed reduction order, so results do not depend on scheduling:
// per-block partial sums (dot, norm and the 16 channel sums of vp and nc) into a small
// workspace, then every block of the update kernel reduces the partials in the same order.
#include <algorithm>

#include "common.cuh"

namespace vdit {
namespace {

constexpr int kThreads = 256;          // a multiple of 16: each thread keeps one latent channel
constexpr int kParts = 128;            // blocks of the statistics kernel
constexpr int kStats = 2 + 2 * 16;     // dot, norm, channel sums of vp, channel sums of nc

__device__ __forceinline__ float neg_candidate(const float* xt, const float* ln, const float* x0, int64_t e, float a,
                                               float inv_t) {
    const float l = ln[e];
    return x0 ? (1.f - a) * l + a * ((xt[e] - x0[e]) * inv_t) : l;
}

__global__ void __launch_bounds__(kThreads) cfg_reuse_stats_kernel(const float* __restrict__ xt,
                                                                   const float* __restrict__ vp,
                                                                   const float* __restrict__ ln,
                                                                   const float* __restrict__ x0, int64_t total,
                                                                   float a, float inv_t, float* __restrict__ part) {
    __shared__ float red[kThreads / 32][kStats];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float dot = 0.f, nn = 0.f, svp = 0.f, snc = 0.f;      // this thread's channel is tid % 16
    for (int64_t e = (int64_t)blockIdx.x * kThreads + tid; e < total; e += (int64_t)gridDim.x * kThreads) {
        const float v = vp[e], c = neg_candidate(xt, ln, x0, e, a, inv_t);
        dot = fmaf(v, c, dot);
        nn = fmaf(c, c, nn);
        svp += v;
        snc += c;
    }
    // lanes l and l + 16 hold the same channel: fold them, then sum all lanes for dot / norm
    const float svp2 = svp + __shfl_xor_sync(0xffffffffu, svp, 16);
    const float snc2 = snc + __shfl_xor_sync(0xffffffffu, snc, 16);
    dot = warp_sum(dot);
    nn = warp_sum(nn);
    if (lane == 0) {
        red[warp][0] = dot;
        red[warp][1] = nn;
    }
    if (lane < 16) {
        red[warp][2 + lane] = svp2;
        red[warp][18 + lane] = snc2;
    }
    __syncthreads();
    if (tid < kStats) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) s += red[w][tid];
        part[blockIdx.x * kStats + tid] = s;
    }
}

__global__ void __launch_bounds__(kThreads) cfg_reuse_apply_kernel(float* __restrict__ xt, const float* __restrict__ vp,
                                                                   const float* __restrict__ ln,
                                                                   const float* __restrict__ x0, int64_t n, float a,
                                                                   float inv_t, float g, float dt, float hf,
                                                                   int zero_star, int nparts,
                                                                   const float* __restrict__ part) {
    __shared__ float st[kStats];
    const int tid = threadIdx.x;
    if (tid < kStats) {
        float s = 0.f;
        for (int p = 0; p < nparts; ++p) s += part[p * kStats + tid];     // fixed order in every block
        st[tid] = s;
    }
    __syncthreads();
    const int ch = tid & 15;
    const float s = zero_star ? fminf(fmaxf(st[0] / fmaxf(st[1], 1e-6f), 0.9f), 1.1f) : 1.f;
    const float dc = (st[2 + ch] - s * st[18 + ch]) / (float)n;        // row mean of delta, channel ch
    const int64_t total = n * 16;
    for (int64_t e = (int64_t)blockIdx.x * kThreads + tid; e < total; e += (int64_t)gridDim.x * kThreads) {
        const float v = vp[e];
        float d = v - s * neg_candidate(xt, ln, x0, e, a, inv_t);
        if (hf != 0.f) d += hf * (d - dc);
        xt[e] -= dt * (v + g * d);
    }
}

__global__ void neg_endpoint_kernel(const float* __restrict__ xt, const float* __restrict__ vn, int64_t total, float t,
                                    float* __restrict__ x0) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < total) x0[e] = xt[e] - t * vn[e];
}

}  // namespace
}  // namespace vdit

using namespace vdit;

extern "C" size_t vdit_cfg_reuse_workspace_bytes(void) { return (size_t)kParts * kStats * sizeof(float); }

extern "C" int vdit_cfg_reuse_euler(float* xt, const float* vp, const float* last_neg, const float* last_neg_x0,
                                    int64_t n, float guidance, float dt, float t_eval, float endpoint_blend,
                                    float hf_gain, int32_t zero_star, void* workspace, size_t workspace_bytes,
                                    vdit_stream_t stream) {
    if (!xt || !vp || !last_neg || n < 0 || !(t_eval > 0.f) || endpoint_blend < 0.f || endpoint_blend > 1.f)
        return VDIT_ERR_ARG;
    if (!workspace || workspace_bytes < vdit_cfg_reuse_workspace_bytes()) return VDIT_ERR_WORKSPACE;
    if (n == 0) return VDIT_OK;
    // without the projection the reference reuses last_neg as it is: no blend, no boost
    const float* x0 = (zero_star && endpoint_blend > 0.f) ? last_neg_x0 : nullptr;
    const float a = x0 ? endpoint_blend : 0.f, hf = zero_star ? hf_gain : 0.f;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* part = static_cast<float*>(workspace);
    cfg_reuse_stats_kernel<<<kParts, kThreads, 0, s>>>(xt, vp, last_neg, x0, n * 16, a, 1.f / t_eval, part);
    const int blocks = (int)std::min<int64_t>((n * 16 + kThreads - 1) / kThreads, 1184);
    cfg_reuse_apply_kernel<<<blocks, kThreads, 0, s>>>(xt, vp, last_neg, x0, n, a, 1.f / t_eval, guidance, dt, hf,
                                                       zero_star, kParts, part);
    count_launches(2);
    return check_launch();
}

extern "C" int vdit_neg_endpoint(const float* xt, const float* v_neg, int64_t n, float t_eval, float* x0,
                                 vdit_stream_t stream) {
    if (!xt || !v_neg || !x0 || n < 0) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    const int64_t total = n * 16;
    neg_endpoint_kernel<<<(unsigned)((total + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(xt, v_neg, total,
                                                                                                        t_eval, x0);
    count_launches(1);
    return check_launch();
}
