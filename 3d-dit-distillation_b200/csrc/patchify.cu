// Patchify on the tensor cores: x[n, d] bf16 = xt[n, 16] fp32 @ w[d, 16]^T fp32.
//
// Both fp32 operands are split into two bf16 parts, hi = bf16(v) and lo = bf16(v - hi), so that
// x = x_hi w_hi + x_hi w_lo + x_lo w_hi up to the dropped x_lo w_lo term and the 16-bit
// significands of the parts (about 2^-16 relative, far below the bf16 rounding of the output).
// With A = [x_hi | x_lo] (rows x 32) and B = [w_hi | w_lo] (channels x 32) the three products are
// three K=16 MMAs into one fp32 accumulator.
//
// A persistent CTA owns one column of 256 output channels, splits its weights into shared memory
// once (16 KB), and walks its share of the 128-row tiles of that column.  Warps 0-3 (thread =
// row) split the tile's 128 input rows into an A buffer, then read back the previous tile's
// accumulator (TMEM lanes 32 warp ..) and store it as bf16 through swizzled 32-row x 64-column
// boxes written by TMA; warp 4 issues the MMAs.  A and the accumulator are double-buffered, so the split of tile t and the store of tile
// t - 1 overlap the MMAs.  Operands use the no-swizzle K-major layout: core matrices of 8 rows x
// 16 bytes, 128 bytes apart along K and 512 bytes apart per 8 rows.  The kernel is bound by the
// output stores.  Waits are bounded; a timeout sets the error word and the CTA skips to its
// teardown.
#include <algorithm>

#include "common.cuh"
#include "tc.cuh"

namespace vdit {
__device__ int g_patchify_error = 0;

namespace {

constexpr int kPtRows = 128;                      // output rows per tile (the MMA's M)
constexpr int kPtCols = 256;                      // output channels per tile (the MMA's N)
constexpr int kPtABytes = kPtRows * 64;           // [x_hi | x_lo] of 128 rows
constexpr int kPtBOff = 0;                        // B: [w_hi | w_lo] of the CTA's 256 channels
constexpr int kPtAOff = kPtCols * 64;
constexpr int kPtBoxOff = kPtAOff + 2 * kPtABytes;
constexpr int kPtBoxBytes = 32 * 128;             // 32 rows x 64 bf16 channels
constexpr int kPtBarOff = kPtBoxOff + 4 * 2 * kPtBoxBytes;
// more shared memory than two CTAs could share: one CTA per SM, which owns all 512 TMEM columns
constexpr int kPtSmem = 1024 + kPtBarOff + 128 > 116 * 1024 ? 1024 + kPtBarOff + 128 : 116 * 1024;
constexpr int kErrPtTimeout = 0x5054;             // "PT": a bounded wait ran out
constexpr uint32_t kPtIdesc = tc::make_idesc(kPtRows, kPtCols, false);

// byte offset of bf16 element k (0..31) of row r in the no-swizzle K-major layout
__device__ __forceinline__ uint32_t pt_off(int r, int k) {
    return (uint32_t)((r >> 3) * 512 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(x), "r"(y)
                 : "memory");
}

// the 8 values hi/lo-split into two 16-byte groups of bf16
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
    float h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const __nv_bfloat16 b = __float2bfloat16_rn(v[j]);
        h[j] = __bfloat162float(b);
        l[j] = v[j] - h[j];
    }
    hi = pack8(h);
    lo = pack8(l);
}

__global__ void __launch_bounds__(160, 1) patchify_tc_kernel(const float* __restrict__ xt, int64_t n,
                                                            const float* __restrict__ w, int d,
                                                            const __grid_constant__ CUtensorMap tm_out) {
    using namespace tc;
    extern __shared__ uint8_t pt_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pt_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kPtBarOff);
    // a_full[2] (128 arrivals), a_empty[2], acc_full[2], acc_empty[2] (128 arrivals)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    auto a_full = [&](int b) { return smem_u32(&bars[b]); };
    auto a_empty = [&](int b) { return smem_u32(&bars[2 + b]); };
    auto acc_full = [&](int b) { return smem_u32(&bars[4 + b]); };
    auto acc_empty = [&](int b) { return smem_u32(&bars[6 + b]); };
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // the CTA's column of 256 channels and its share of the row tiles
    const int col_tiles = (d + kPtCols - 1) / kPtCols;
    const int64_t row_tiles = (n + kPtRows - 1) / kPtRows;
    const int ct = (int)(blockIdx.x % col_tiles);
    const int cpc = ((int)gridDim.x - ct + col_tiles - 1) / col_tiles;      // CTAs on this column
    const int64_t rt0 = blockIdx.x / col_tiles;
    // row r = 32 warp + lane of a tile (warps 0-3): its 16 inputs, loaded one tile ahead (the first
    // before the weight split, later ones while the previous tile is stored)
    const int r = warp * 32 + lane;
    auto load_row = [&](int64_t rt, float4 (&x)[4]) {
        const int64_t row = rt * kPtRows + r;
#pragma unroll
        for (int q = 0; q < 4; ++q)
            x[q] = (rt < row_tiles && row < n) ? __ldg(reinterpret_cast<const float4*>(xt + row * 16) + q)
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    float4 xn[4];
    if (warp < 4) load_row(rt0, xn);

    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(a_full(b), 128);
            mbar_init(a_empty(b), 1);
            mbar_init(acc_full(b), 1);
            mbar_init(acc_empty(b), 128);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_out)) : "memory");
    }
    // B: the split weight of the CTA's 256 channels, channel ct * 256 + i at row i (channels past
    // d zero), all threads; each thread loads two channels' weights before splitting them
    for (int i0 = tid; i0 < kPtCols; i0 += 2 * (int)blockDim.x) {
        float4 wl[2][4];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int c = ct * kPtCols + i0 + u * (int)blockDim.x;
#pragma unroll
            for (int q = 0; q < 4; ++q)
                wl[u][q] = (i0 + u * (int)blockDim.x < kPtCols && c < d)
                               ? __ldg(reinterpret_cast<const float4*>(w + (int64_t)c * 16) + q)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int c = i0 + u * (int)blockDim.x;
            if (c >= kPtCols) break;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const float4 a = wl[u][2 * half], b = wl[u][2 * half + 1];
                const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                uint4 hi, lo;
                split8(v, hi, lo);
                *reinterpret_cast<uint4*>(sm + kPtBOff + pt_off(c, 8 * half)) = hi;
                *reinterpret_cast<uint4*>(sm + kPtBOff + pt_off(c, 16 + 8 * half)) = lo;
            }
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ---------------- MMA issuer: per tile acc = A_hi B_hi^T + A_hi B_lo^T + A_lo B_hi^T
        const uint64_t a0 = make_desc(smem_u32(sm + kPtAOff), 128, 512, 0);
        const uint64_t b0 = make_desc(smem_u32(sm + kPtBOff), 128, 512, 0);
        auto wait = [&](uint32_t bar, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, &g_patchify_error, kErrPtTimeout));
        };
        int lt = 0;
        for (int64_t rt = rt0; rt < row_tiles; rt += cpc, ++lt) {
            const int buf = lt & 1;
            if (!wait(a_full(buf), (lt >> 1) & 1)) break;
            if (lt >= 2 && !wait(acc_empty(buf), ((lt >> 1) - 1) & 1)) break;
            tc_fence_after();
            const uint64_t a = a0 + (uint64_t)(buf * (kPtABytes >> 4));
            const uint64_t b = b0;
            const uint32_t acc = tmem + buf * kPtCols;
            tc_mma_elect(acc, a, b, kPtIdesc, 0u);                         // hi x hi
            tc_mma_elect(acc, a, b + (256 >> 4), kPtIdesc, 1u);            // hi x lo
            tc_mma_elect(acc, a + (256 >> 4), b, kPtIdesc, 1u);            // lo x hi
            tc_commit_elect(a_empty(buf));
            tc_commit_elect(acc_full(buf));
        }
    } else {
        // ---------------- warps 0-3: split the inputs, then store the previous tile
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        int lt = 0, nstore = 0;
        bool ok = true;
        int64_t prev = -1;
        auto epilogue = [&](int64_t t, int l) {
            const int buf = l & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(acc_full(buf), (l >> 1) & 1, abort_flag, &g_patchify_error,
                                                   kErrPtTimeout)))
                return false;
            tc_fence_after();
            const int64_t row0 = t * kPtRows + warp * 32;
            const int col0 = ct * kPtCols;
#pragma unroll 1
            for (int c = 0; c < kPtCols / 64; ++c, ++nstore) {
                float v[64];
                tmem_ld32(tmem + buf * kPtCols + c * 64 + lane_off, v);
                tmem_ld32(tmem + buf * kPtCols + c * 64 + 32 + lane_off, v + 32);
                tmem_wait_ld();
                uint8_t* box = sm + kPtBoxOff + (warp * 2 + (nstore & 1)) * kPtBoxBytes;
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                __syncwarp();
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    *reinterpret_cast<uint4*>(box + lane * 128 + ((q ^ (lane & 7)) << 4)) = pack8(v + q * 8);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    // boxes starting past n or d are skipped; the map clips the ones that cross
                    if (row0 < n && col0 + c * 64 < d) tma_store_2d(&tm_out, smem_u32(box), col0 + c * 64, (int)row0);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            tc_fence_before();
            mbar_arrive(acc_empty(buf));
            return true;
        };
        for (int64_t t = rt0; ok && t < row_tiles; t += cpc, ++lt) {
            const int buf = lt & 1;
            if (lt >= 2 && !__all_sync(0xffffffffu, mbar_wait(a_empty(buf), ((lt >> 1) - 1) & 1, abort_flag,
                                                              &g_patchify_error, kErrPtTimeout))) {
                ok = false;
                break;
            }
            float v[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[4 * q] = xn[q].x; v[4 * q + 1] = xn[q].y; v[4 * q + 2] = xn[q].z; v[4 * q + 3] = xn[q].w;
            }
            load_row(t + cpc, xn);
            uint8_t* ab = sm + kPtAOff + buf * kPtABytes;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint4 hi, lo;
                split8(v + 8 * h, hi, lo);
                *reinterpret_cast<uint4*>(ab + pt_off(r, 8 * h)) = hi;
                *reinterpret_cast<uint4*>(ab + pt_off(r, 16 + 8 * h)) = lo;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(a_full(buf));
            if (prev >= 0 && !epilogue(prev, lt - 1)) {
                ok = false;
                break;
            }
            prev = t;
        }
        if (ok && prev >= 0) epilogue(prev, lt - 1);
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // stores done before exit
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

bool make_out_map(CUtensorMap* map, void* base, int64_t rows, int cols) {
    auto fn = tc::encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {64, 32};
    cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

}  // namespace

int patchify_error_word(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_patchify_error, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    if (clear) {
        int z = 0;
        if (cudaMemcpyToSymbol(g_patchify_error, &z, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    }
    return v;
}

}  // namespace vdit

using namespace vdit;

extern "C" int vdit_patchify(const float* xt, int64_t n, const float* w, int32_t d, void* x_out, vdit_stream_t stream) {
    if (n < 0 || d <= 0 || d % 8 || !xt || !w || !x_out) return VDIT_ERR_ARG;
    if (!aligned16(xt) || !aligned16(w) || !aligned16(x_out)) return VDIT_ERR_ALIGN;
    if (n == 0) return VDIT_OK;
    if (n > INT32_MAX) return VDIT_ERR_UNSUPPORTED;                 // TMA row coordinates are 32-bit
    static bool attr_set[64] = {false};
    static int sms[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        if (e != cudaSuccess) record_cuda_error(e);
        return VDIT_ERR_LAUNCH;
    }
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(patchify_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPtSmem);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return VDIT_ERR_LAUNCH;
        }
        attr_set[dev] = true;
    }
    CUtensorMap mo;
    if (!make_out_map(&mo, x_out, n, d)) return VDIT_ERR_DRIVER;
    const int64_t tiles = ((n + kPtRows - 1) / kPtRows) * ((d + kPtCols - 1) / kPtCols);
    // every column of 256 channels gets at least one CTA
    const unsigned grid = (unsigned)std::max<int64_t>(std::min<int64_t>(tiles, sms[dev]), (d + kPtCols - 1) / kPtCols);
    patchify_tc_kernel<<<grid, 160, kPtSmem, static_cast<cudaStream_t>(stream)>>>(xt, n, w, d, mo);
    count_launches(1);
    return check_launch();
}
