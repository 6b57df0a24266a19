// Depthwise 27-tap submanifold sparse conv (the block's ffn_conv) with an
// optional fused SwiGLU epilogue.  HBM-bound gather: every output row reads
// its present neighbours' rows; rows are visited in lexicographic voxel order,
// so a neighbour row was fetched moments earlier by a nearby warp and comes
// from L2 (DRAM sees about one read of the input and one write of the output).
//
// Mapping: one warp = one output row x one 256-channel tile; lane l owns 8
// output channels (16-byte vectors).  The 27 neighbour indices of the row are
// read by lanes 0..26 in one coalesced load, a ballot gives the valid-tap mask
// and the warp walks only the valid taps (warp-uniform, no divergence),
// issuing the loads of up to kBatch taps before their FMAs.  The next row's
// indices are fetched while the current row is accumulated.  fp32 weights of
// the tile live in shared memory; accumulation is fp32.
#include "common.cuh"

namespace vdit {
namespace {

constexpr int kVec = 8;            // channels per lane (one 16-byte bf16 vector)
constexpr int kLanesTile = 32;     // lanes per row -> 256 output channels per tile
constexpr int kTile = kLanesTile * kVec;
constexpr int kWarps = 8;
constexpr int kRowsPerWarp = 8;    // consecutive rows per warp per CTA
constexpr int kBatch = 4;          // taps whose loads are in flight together

__device__ __forceinline__ void fma8(float* acc, const uint4& u, const float* __restrict__ w) {
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float4 w0 = *reinterpret_cast<const float4*>(w);
    const float4 w1 = *reinterpret_cast<const float4*>(w + 4);
    float2 f;
    f = __bfloat1622float2(p[0]); acc[0] = fmaf(f.x, w0.x, acc[0]); acc[1] = fmaf(f.y, w0.y, acc[1]);
    f = __bfloat1622float2(p[1]); acc[2] = fmaf(f.x, w0.z, acc[2]); acc[3] = fmaf(f.y, w0.w, acc[3]);
    f = __bfloat1622float2(p[2]); acc[4] = fmaf(f.x, w1.x, acc[4]); acc[5] = fmaf(f.y, w1.y, acc[5]);
    f = __bfloat1622float2(p[3]); acc[6] = fmaf(f.x, w1.z, acc[6]); acc[7] = fmaf(f.y, w1.w, acc[7]);
}

// FUSE = false: out[n, c] over channel tile [t0, t0+kTile)
// FUSE = true : out[n, c/2 + ..] = silu(y[:, c/2 + j]) * y[:, j] for j in the tile
template <bool FUSE>
__global__ void __launch_bounds__(kWarps * 32, 3) dwconv27_kernel(const __nv_bfloat16* __restrict__ h, int64_t n,
                                                                  int c, const int32_t* __restrict__ idx,
                                                                  const float* __restrict__ w,
                                                                  const float* __restrict__ b,
                                                                  __nv_bfloat16* __restrict__ out) {
    constexpr int G = FUSE ? 2 : 1;
    extern __shared__ __align__(16) float smem[];
    float* ws = smem;                        // [27][G][kTile]
    float* bs = smem + 27 * G * kTile;       // [G][kTile]
    const int half = c / 2;
    const int width = FUSE ? half : c;
    const int t0 = blockIdx.x * kTile;
    for (int t = threadIdx.x; t < 27 * G * kTile; t += blockDim.x) {
        const int j = t % kTile, g = (t / kTile) % G, d = t / (kTile * G);
        ws[t] = (t0 + j < width) ? w[(int64_t)d * c + t0 + g * half + j] : 0.f;
    }
    for (int t = threadIdx.x; t < G * kTile; t += blockDim.x)
        bs[t] = (t0 + t % kTile < width) ? b[t0 + (t / kTile) * half + t % kTile] : 0.f;
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ch = t0 + lane * kVec;
    const bool active = ch < width;                  // the last tile may be partial
    const int64_t row0 = ((int64_t)blockIdx.y * kWarps + warp) * kRowsPerWarp;
    const int64_t row_end = min(n, row0 + kRowsPerWarp);
    if (row0 >= n) return;
    int my = (lane < 27) ? __ldg(idx + row0 * 27 + lane) : -1;
    for (int64_t row = row0; row < row_end; ++row) {
        const int nxt = (lane < 27 && row + 1 < row_end) ? __ldg(idx + (row + 1) * 27 + lane) : -1;
        unsigned mask = __ballot_sync(0xffffffffu, my >= 0);
        float acc[G][kVec];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < kVec; ++j) acc[g][j] = bs[g * kTile + lane * kVec + j];
        while (mask) {
            int taps[kBatch];
            uint4 va[kBatch], vg[kBatch];
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                taps[k] = -1;
                if (mask) {                                   // warp-uniform
                    const int d = __ffs(mask) - 1;
                    mask &= mask - 1;
                    taps[k] = d;
                    const int src = __shfl_sync(0xffffffffu, my, d);
                    const __nv_bfloat16* hr = h + (int64_t)src * c;
                    if (active) {
                        va[k] = __ldg(reinterpret_cast<const uint4*>(hr + ch));
                        if (FUSE) vg[k] = __ldg(reinterpret_cast<const uint4*>(hr + half + ch));
                    } else {
                        va[k] = make_uint4(0, 0, 0, 0);
                        vg[k] = make_uint4(0, 0, 0, 0);
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                if (taps[k] < 0) break;
                const float* wd = ws + taps[k] * G * kTile + lane * kVec;
                fma8(acc[0], va[k], wd);
                if (FUSE) fma8(acc[G - 1], vg[k], wd + kTile);
            }
        }
        float o[kVec];
        if (FUSE) {
#pragma unroll
            for (int j = 0; j < kVec; ++j) {
                // the reference stores the conv output in bf16 before the SwiGLU reads it
                const float a = bf2f(f2bf(acc[0][j]));
                const float g = bf2f(f2bf(acc[G - 1][j]));
                o[j] = silu(g) * a;
            }
            if (active) store8(out + row * half + ch, o);
        } else {
#pragma unroll
            for (int j = 0; j < kVec; ++j) o[j] = acc[0][j];
            if (active) store8(out + row * c + ch, o);
        }
        my = nxt;
    }
}

template <bool FUSE>
int launch_dw(const void* h, int64_t n, int32_t c, const int32_t* idx, const float* w, const float* b, void* out,
              cudaStream_t s) {
    const int width = FUSE ? c / 2 : c;
    if (width % kVec) return VDIT_ERR_UNSUPPORTED;
    const size_t sm = (size_t)(27 + 1) * (FUSE ? 2 : 1) * kTile * sizeof(float);
    static bool configured = false;
    if (!configured) {
        const cudaError_t e = cudaFuncSetAttribute(dwconv27_kernel<FUSE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return VDIT_ERR_LAUNCH;
        }
        configured = true;
    }
    const int64_t rows_per_cta = (int64_t)kWarps * kRowsPerWarp;
    dim3 grid((width + kTile - 1) / kTile, (unsigned)((n + rows_per_cta - 1) / rows_per_cta));
    dwconv27_kernel<FUSE><<<grid, kWarps * 32, sm, s>>>(static_cast<const __nv_bfloat16*>(h), n, c, idx, w, b,
                                                         static_cast<__nv_bfloat16*>(out));
    return VDIT_OK;
}

}  // namespace
}  // namespace vdit

using namespace vdit;

extern "C" int vdit_dwconv27(const void* h, int64_t n, int32_t c, const int32_t* idx, const float* w, const float* b,
                             void* out, int32_t fuse_swiglu, vdit_stream_t stream) {
    if (n < 0 || c <= 0 || !h || !idx || !w || !b || !out) return VDIT_ERR_ARG;
    if (fuse_swiglu && (c % 2)) return VDIT_ERR_ARG;
    if (!aligned16(h) || !aligned16(out)) return VDIT_ERR_ALIGN;
    if (n == 0) return VDIT_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int rc = fuse_swiglu ? launch_dw<true>(h, n, c, idx, w, b, out, s) : launch_dw<false>(h, n, c, idx, w, b, out, s);
    if (rc != VDIT_OK) return rc;
    count_launches(1);
    return check_launch();
}
