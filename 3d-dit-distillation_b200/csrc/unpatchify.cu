// Output projection of the unpatchify step on the tensor cores at fp32 accuracy:
// out[m, 16] fp32 = y[m, d] (bf16, the modulated rows) @ w[16, d]^T with fp32 weights.
//
// Each weight is split into three bf16 parts, hi = bf16(w), mid = bf16(w - hi), lo = bf16(w - hi -
// mid): both differences are exact in fp32, and hi + mid + lo carries w's 24-bit significand.  The
// split weight w3 [48, d] (rows 16 p + o hold part p of output o) is made once per weight by
// vdit_split_weight3.  Every product y * part (bf16 x bf16) is exact in the fp32 accumulator, so one
// M=128, N=48 MMA chain over d gives the three partial sums of each output, which the epilogue adds
// (lo + mid first).
//
// A CTA takes 128 rows.  Lane 0 of warp 0 streams 64-column chunks of the rows (128 x 128 bytes)
// and of w3 (48 x 128 bytes) into a six-stage ring with TMA (128-byte swizzle; rows past m and
// columns past d read as zeros); warp 1 issues each chunk's four K=16 MMAs into a 48-column TMEM
// accumulator and frees the stage with a commit; warps 0-3 read the accumulator back (warp q: rows
// 32q .. 32q + 31) and store each row's 16 outputs.  The rows are read once from HBM: the kernel is
// bound by that read.  Waits are bounded: a timeout sets the error word and the CTA skips to its
// teardown.
#include "common.cuh"
#include "tc.cuh"

namespace vdit {
__device__ int g_unpatch_error = 0;

namespace {

constexpr int kPrRows = 128;                          // rows per CTA (the MMA's M)
constexpr int kPrK = 64;                              // columns per chunk (128 bytes of bf16)
constexpr int kPrN = 48;                              // hi, mid and lo parts of 16 outputs
constexpr int kPrStages = 6;
constexpr int kPrABytes = kPrRows * 128;
constexpr int kPrStageBytes = kPrABytes + kPrN * 128;  // 22 KB, a multiple of 1024
constexpr int kPrBarOff = kPrStages * kPrStageBytes;
constexpr int kPrSmem = 1024 + kPrBarOff + 256;       // 1024: alignment slack
constexpr int kErrPrTimeout = 0x5550;                 // "UP": a bounded wait ran out
static_assert(kPrStageBytes % 1024 == 0, "stage alignment");
static_assert((2 * kPrStages + 1) * 8 + 8 <= 256, "barrier area");

__global__ void split3_kernel(const float* __restrict__ w, int rows, int d, __nv_bfloat16* __restrict__ w3) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * d) return;
    const int64_t o = i / d, c = i - o * d;
    float r = w[i];
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        const __nv_bfloat16 b = __float2bfloat16_rn(r);
        r -= __bfloat162float(b);
        w3[(p * rows + o) * d + c] = b;
    }
}

__global__ void __launch_bounds__(128, 1) unpatchify_project_kernel(const __grid_constant__ CUtensorMap tm_y,
                                                                   const __grid_constant__ CUtensorMap tm_w,
                                                                   int64_t m, int d, float* __restrict__ out) {
    using namespace tc;
    extern __shared__ uint8_t pr_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pr_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kPrBarOff);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kPrStages + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = (int64_t)blockIdx.x * kPrRows;
    const int nk = (d + kPrK - 1) / kPrK;
    auto full = [&](int s) { return smem_u32(&bars[s]); };
    auto empty = [&](int s) { return smem_u32(&bars[kPrStages + s]); };
    const uint32_t done = smem_u32(&bars[2 * kPrStages]);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPrStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_y)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 64;" ::"r"(smem_u32(tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer
        if (lane == 0) {
            for (int k = 0; k < nk; ++k) {
                const int s = k % kPrStages;
                if (k >= kPrStages &&
                    !mbar_wait(empty(s), ((k / kPrStages) - 1) & 1, abort_flag, &g_unpatch_error, kErrPrTimeout))
                    break;
                const uint32_t stg = smem_u32(sm + s * kPrStageBytes);
                mbar_expect_tx(full(s), (uint32_t)kPrStageBytes);
                tma_load_2d(stg, &tm_y, k * kPrK, (int)row0, full(s));
                tma_load_2d(stg + kPrABytes, &tm_w, k * kPrK, 0, full(s));
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (converged warp, elected lane)
        const uint64_t a0 = make_desc(smem_u32(sm), 16, 1024, kSw128);
        const uint64_t b0 = make_desc(smem_u32(sm + kPrABytes), 16, 1024, kSw128);
        constexpr uint32_t kIdesc = make_idesc(kPrRows, kPrN, false);
        bool ok = true;
        for (int k = 0; k < nk; ++k) {
            const int s = k % kPrStages;
            if (!__all_sync(0xffffffffu, mbar_wait(full(s), (k / kPrStages) & 1, abort_flag, &g_unpatch_error,
                                                   kErrPrTimeout))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint64_t so = (uint64_t)(s * (kPrStageBytes >> 4));
#pragma unroll
            for (int kk = 0; kk < kPrK / 16; ++kk)
                tc_mma_elect(tmem, a0 + so + kk * 2, b0 + so + kk * 2, kIdesc, (k > 0 || kk > 0) ? 1u : 0u);
            tc_commit_elect(empty(s));
        }
        if (ok) tc_commit_elect(done);
    }

    // ---------------- epilogue: warp q reads TMEM lanes 32q .. 32q + 31 (the tile's rows)
    if (__all_sync(0xffffffffu, mbar_wait(done, 0, abort_flag, &g_unpatch_error, kErrPrTimeout))) {
        tc_fence_after();
        float v[64];
        const uint32_t ta = tmem + ((uint32_t)(32 * warp) << 16);
        tmem_ld32(ta, v);
        tmem_ld32(ta + 32, v + 32);
        tmem_wait_ld();
        const int64_t row = row0 + 32 * warp + lane;
        if (row < m) {
            float4* dst = reinterpret_cast<float4*>(out + row * 16);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = (v[32 + 4 * q + e] + v[16 + 4 * q + e]) + v[4 * q + e];
                dst[q] = make_float4(o[0], o[1], o[2], o[3]);
            }
        }
    } else if (warp == 0 && lane == 0) {
        // a wait ran out: let the loads still in flight land before the CTA leaves
        volatile int no_abort = 0;
        for (int k = 0; k < nk && k < kPrStages; ++k) {
            const int kl = nk - 1 - k;            // the last stages issued
            mbar_wait(full(kl % kPrStages), (kl / kPrStages) & 1, &no_abort, &g_unpatch_error, kErrPrTimeout);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 64;" ::"r"(tmem));
    }
}

// 2-D bf16 tensor map over [rows, cols] (row stride ld elements), box {64 columns, box_rows rows},
// 128-byte swizzle, zero fill outside
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int cols, int64_t ld, int box_rows) {
    auto fn = tc::encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)kPrK, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int unpatch_error_word(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_unpatch_error, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    if (clear) {
        int z = 0;
        if (cudaMemcpyToSymbol(g_unpatch_error, &z, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    }
    return v;
}

}  // namespace vdit

using namespace vdit;

extern "C" int vdit_split_weight3(const float* w, int32_t rows, int32_t d, void* w3, vdit_stream_t stream) {
    if (rows < 1 || d < 1 || !w || !w3) return VDIT_ERR_ARG;
    const int64_t n = (int64_t)rows * d;
    split3_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        w, rows, d, static_cast<__nv_bfloat16*>(w3));
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_unpatchify_project(const void* y, int64_t m, int32_t d, const void* w3, float* out,
                                       vdit_stream_t stream) {
    if (m < 0 || d < 8 || d % 8 || !y || !w3 || !out) return VDIT_ERR_ARG;
    if (!aligned16(y) || !aligned16(w3) || !aligned16(out)) return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    if (m > INT32_MAX) return VDIT_ERR_UNSUPPORTED;          // TMA row coordinates are 32-bit
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        if (e != cudaSuccess) record_cuda_error(e);
        return VDIT_ERR_LAUNCH;
    }
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(unpatchify_project_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrSmem);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return VDIT_ERR_LAUNCH;
        }
        attr_set[dev] = true;
    }
    CUtensorMap my, mw;
    if (!make_map(&my, y, m, d, d, kPrRows) || !make_map(&mw, w3, kPrN, d, d, kPrN)) return VDIT_ERR_DRIVER;
    const int64_t tiles = (m + kPrRows - 1) / kPrRows;
    unpatchify_project_kernel<<<(unsigned)tiles, 128, kPrSmem, static_cast<cudaStream_t>(stream)>>>(my, mw, m, d, out);
    count_launches(1);
    return check_launch();
}
