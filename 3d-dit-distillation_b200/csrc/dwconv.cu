// Depthwise 27-tap submanifold sparse conv (the block's ffn_conv) with an
// optional fused SwiGLU epilogue.  HBM-bound gather: each output row reads
// its present neighbours' rows (16-byte vectors, fp32 accumulation with the
// fp32 weights staged in shared memory).  Rows are visited in the
// lexicographic voxel order, so the neighbours of a row group were read by
// nearby blocks moments earlier and come from L2; DRAM sees ~one read of the
// input and one write of the output.
#include "common.cuh"

namespace vdit {
namespace {

constexpr int kVec = 8;          // channels per thread (one 16-byte bf16 vector)
constexpr int kThreads = 256;
constexpr int kRowIters = 4;     // row slots visited per thread

// FUSE = false: out[n, c]  (tile = TPR*8 channels)
// FUSE = true : out[n, c/2] = silu(y[:, c/2 + j]) * y[:, j]  (tile = TPR*8 output channels,
//               needing the two conv channel groups j and c/2 + j)
template <bool FUSE, int TPR>
__global__ void __launch_bounds__(kThreads) dwconv27_kernel(const __nv_bfloat16* __restrict__ h, int64_t n, int c,
                                                            const int32_t* __restrict__ idx,
                                                            const float* __restrict__ w, const float* __restrict__ b,
                                                            __nv_bfloat16* __restrict__ out) {
    constexpr int kTile = TPR * kVec;            // output channels per block
    constexpr int kGroups = FUSE ? 2 : 1;
    constexpr int kRowsPerPass = kThreads / TPR;
    __shared__ __align__(16) float ws[27 * kGroups * kTile];
    __shared__ __align__(16) float bs[kGroups * kTile];

    const int half = c / 2;
    const int tile0 = blockIdx.x * kTile;        // first output channel of this tile
    // stage weights: ws[(d*kGroups + g)*kTile + j] = w[d, tile0 + g*half + j]
    for (int t = threadIdx.x; t < 27 * kGroups * kTile; t += kThreads) {
        int j = t % kTile, g = (t / kTile) % kGroups, d = t / (kTile * kGroups);
        ws[t] = w[(int64_t)d * c + tile0 + g * half + j];
    }
    for (int t = threadIdx.x; t < kGroups * kTile; t += kThreads) {
        int j = t % kTile, g = t / kTile;
        bs[t] = b[tile0 + g * half + j];
    }
    __syncthreads();

    const int lane_c = (threadIdx.x % TPR) * kVec;   // channel offset inside the tile
    const int slot = threadIdx.x / TPR;
    const int ch_a = tile0 + lane_c;                 // input channel of group 0
    const int ch_g = tile0 + half + lane_c;          // input channel of group 1 (FUSE)
    const int out_w = FUSE ? half : c;

    for (int it = 0; it < kRowIters; ++it) {
        const int64_t row = ((int64_t)blockIdx.y * kRowIters + it) * kRowsPerPass + slot;
        if (row >= n) break;
        float acc[kGroups][kVec];
#pragma unroll
        for (int g = 0; g < kGroups; ++g)
#pragma unroll
            for (int j = 0; j < kVec; ++j) acc[g][j] = bs[g * kTile + lane_c + j];
        const int32_t* ir = idx + row * 27;
#pragma unroll
        for (int d0 = 0; d0 < 27; d0 += 9) {
            int nb[9];
#pragma unroll
            for (int k = 0; k < 9; ++k) nb[k] = __ldg(ir + d0 + k);
            uint4 va[9], vg[9];
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                if (nb[k] >= 0) {
                    const __nv_bfloat16* hr = h + (int64_t)nb[k] * c;
                    va[k] = __ldg(reinterpret_cast<const uint4*>(hr + ch_a));
                    if (FUSE) vg[k] = __ldg(reinterpret_cast<const uint4*>(hr + ch_g));
                }
            }
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                if (nb[k] < 0) continue;
                const int d = d0 + k;
#pragma unroll
                for (int g = 0; g < kGroups; ++g) {
                    const uint4 u = g == 0 ? va[k] : vg[k];
                    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
                    const float4 w0 = *reinterpret_cast<const float4*>(&ws[(d * kGroups + g) * kTile + lane_c]);
                    const float4 w1 = *reinterpret_cast<const float4*>(&ws[(d * kGroups + g) * kTile + lane_c + 4]);
                    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float2 f = __bfloat1622float2(p[j]);
                        acc[g][2 * j] = fmaf(f.x, wv[2 * j], acc[g][2 * j]);
                        acc[g][2 * j + 1] = fmaf(f.y, wv[2 * j + 1], acc[g][2 * j + 1]);
                    }
                }
            }
        }
        float o[kVec];
        if (FUSE) {
#pragma unroll
            for (int j = 0; j < kVec; ++j) {
                // the reference stores the conv output in bf16 before the SwiGLU reads it
                float a = bf2f(f2bf(acc[0][j]));
                float g = bf2f(f2bf(acc[kGroups - 1][j]));
                o[j] = silu(g) * a;
            }
        } else {
#pragma unroll
            for (int j = 0; j < kVec; ++j) o[j] = acc[0][j];
        }
        store8(out + row * out_w + tile0 + lane_c, o);
    }
}

}  // namespace
}  // namespace vdit

using namespace vdit;

template <bool FUSE, int TPR>
static void launch_dw(const void* h, int64_t n, int32_t c, const int32_t* idx, const float* w, const float* b, void* out,
                      cudaStream_t s) {
    constexpr int rows_per_block = kRowIters * (kThreads / TPR);
    const int width = FUSE ? c / 2 : c;
    dim3 grid(width / (TPR * kVec), (unsigned)((n + rows_per_block - 1) / rows_per_block));
    dwconv27_kernel<FUSE, TPR><<<grid, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(h), n, c, idx, w, b,
                                                          static_cast<__nv_bfloat16*>(out));
}

template <bool FUSE>
static int dispatch_dw(const void* h, int64_t n, int32_t c, const int32_t* idx, const float* w, const float* b,
                       void* out, cudaStream_t s) {
    const int width = FUSE ? c / 2 : c;
    if (width % kVec) return VDIT_ERR_UNSUPPORTED;
    const int vecs = width / kVec;
    // widest tile (threads per row) that divides the row; weights of one tile fit in static smem
    if (vecs % 16 == 0) launch_dw<FUSE, 16>(h, n, c, idx, w, b, out, s);
    else if (vecs % 8 == 0) launch_dw<FUSE, 8>(h, n, c, idx, w, b, out, s);
    else if (vecs % 4 == 0) launch_dw<FUSE, 4>(h, n, c, idx, w, b, out, s);
    else if (vecs % 2 == 0) launch_dw<FUSE, 2>(h, n, c, idx, w, b, out, s);
    else launch_dw<FUSE, 1>(h, n, c, idx, w, b, out, s);
    return VDIT_OK;
}

extern "C" int vdit_dwconv27(const void* h, int64_t n, int32_t c, const int32_t* idx, const float* w, const float* b,
                             void* out, int32_t fuse_swiglu, vdit_stream_t stream) {
    if (n < 0 || c <= 0 || !h || !idx || !w || !b || !out) return VDIT_ERR_ARG;
    if (fuse_swiglu && (c % 2)) return VDIT_ERR_ARG;
    if (!aligned16(h) || !aligned16(out)) return VDIT_ERR_ALIGN;
    if (n == 0) return VDIT_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int rc = fuse_swiglu ? dispatch_dw<true>(h, n, c, idx, w, b, out, s) : dispatch_dw<false>(h, n, c, idx, w, b, out, s);
    if (rc != VDIT_OK) return rc;
    count_launches(1);
    return check_launch();
}
