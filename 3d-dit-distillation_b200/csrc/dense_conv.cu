// Dense 27-tap submanifold sparse conv on tcgen05 tensor cores (implicit GEMM):
//   out[n, co] = b[co] + sum_d sum_ci W[d, co, ci] * f[idx[n, d], ci]
// M = voxels (two 128-row tiles per CTA sharing every weight tile), N = output
// channels (256 per CTA; one TMEM accumulator of 256 fp32 columns per M tile,
// 512 columns in all), K = taps x input channels (64 per step).  Sharing the
// weight tile between 256 rows halves the weight stream from L2, which bounds
// the one-tile form.
// Warps 0..7 gather the A rows f[idx[n,d], k0:k0+64] with cp.async (eight
// lanes per row, 16-byte copies into the 128B-swizzled K-major layout the MMA reads;
// absent neighbours copy zero bytes and read as zeros), warp 8 loads the weight
// tile W[d, co0:co0+256, k0:k0+64] with TMA (128B swizzle), warp 9 issues the
// MMAs.  A 3-stage ring overlaps gathers, weight loads and MMAs: a gather thread
// marks stage i full as soon as its copies for stage i have landed (checked after it
// issued stage i+1), so the MMAs of two stages can be queued on the tensor core while
// the next gather is in flight (marking stage i only after issuing stage i+2 waited
// for the MMAs of stage i-1 and left the tensor core idle at every hand-off).  Taps that no
// row of the CTA has are skipped.  Warps 0..7 then drain TMEM (warp w: tile
// w/4, lane quarter w%4), add the bias and store bf16.  All mbarrier waits are
// bounded (error word + CTA abort flag).
#include <string.h>

#include "common.cuh"
#include "tc.cuh"

namespace vdit {

__device__ int g_dense_error = 0;

namespace dconv {

using namespace tc;

constexpr int BM = 128, MT = 2, ROWS = BM * MT, BN = 256, BK = 64, S = 3;
constexpr int GATHER_WARPS = ROWS / 32;               // 8
constexpr int THREADS = (GATHER_WARPS + 2) * 32;      // + TMA warp + MMA warp
constexpr int kErr = 0x4443;   // "DC": a bounded wait of the dense conv kernel ran out

struct __align__(1024) Smem {
    uint8_t a[S][MT][BM * 128];
    uint8_t b[S][BN * 128];
    int32_t idx[ROWS * 27];
    uint64_t full_a[S], full_b[S], empty[S], acc_full;
    uint32_t tmem_slot;
    int abort_flag;
    unsigned tapmask;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

struct TapWalk {   // iteration -> (tap, k-chunk) over the set bits of the tap mask
    unsigned rem;
    int tap, kc, nkc;
    __device__ __forceinline__ void init(unsigned m, int n) {
        rem = m;
        tap = __ffs(m) - 1;
        kc = 0;
        nkc = n;
    }
    __device__ __forceinline__ void next() {
        if (++kc == nkc) {
            kc = 0;
            rem &= rem - 1;
            tap = __ffs(rem) - 1;
        }
    }
};

__global__ void __launch_bounds__(THREADS, 1) dense_conv27_kernel(const __grid_constant__ CUtensorMap tmW,
                                                                  const __nv_bfloat16* __restrict__ f, int64_t n,
                                                                  int cin, int cout, const int32_t* __restrict__ idx,
                                                                  const float* __restrict__ bias,
                                                                  __nv_bfloat16* __restrict__ out) {
    extern __shared__ uint8_t raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t row0 = (int64_t)blockIdx.x * ROWS;
    const int co0 = blockIdx.y * BN;
    const int nrows = (int)min((int64_t)ROWS, n - row0);
    volatile int* abort_flag = &sm.abort_flag;

    if (tid == 0) {
        sm.tapmask = 0;
        sm.abort_flag = 0;
    }
    for (int t = tid; t < ROWS * 27; t += THREADS) sm.idx[t] = (t < nrows * 27) ? __ldg(idx + row0 * 27 + t) : -1;
    __syncthreads();
    {
        unsigned m = 0;
        for (int t = tid; t < ROWS * 27; t += THREADS)
            if (sm.idx[t] >= 0) m |= 1u << (t % 27);
        m = __reduce_or_sync(0xffffffffu, m);
        if (lane == 0) atomicOr(&sm.tapmask, m);
    }
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&sm.full_a[s]), ROWS);
            mbar_init(smem_u32(&sm.full_b[s]), 1);
            mbar_init(smem_u32(&sm.empty[s]), 1);
        }
        mbar_init(smem_u32(&sm.acc_full), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    }
    if (warp == GATHER_WARPS + 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&sm.tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_slot;
    const unsigned mask = sm.tapmask;
    const int nkc = cin / BK;
    const int n_iter = __popc(mask) * nkc;

    if (warp < GATHER_WARPS) {
        // ------------------------------------------------------------ A gather
        // thread t copies 16-byte chunk t%8 of rows t/8 + 32k (k = 0..7): the eight lanes of
        // a group cover one row's 128 contiguous bytes, so a warp instruction moves four
        // whole rows and no 32-byte sector is fetched twice
        const int r = tid;                                 // the row this thread drains later
        const int mt = r / BM;
        const int ch = tid & 7, rb = tid >> 3;
        TapWalk tw;
        tw.init(mask, nkc);
        int i = 0;
        for (; i < n_iter; ++i, tw.next()) {
            const int s = i % S;
            if (i >= S && !mbar_wait(smem_u32(&sm.empty[s]), ((i / S) - 1) & 1, abort_flag, &g_dense_error, kErr))
                break;
#pragma unroll
            for (int k = 0; k < ROWS / 32; ++k) {
                const int rr = rb + 32 * k, rt = rr % BM;
                const int src = sm.idx[rr * 27 + tw.tap];
                const __nv_bfloat16* p = f + (int64_t)(src >= 0 ? src : 0) * cin + tw.kc * BK + ch * 8;
                cp_async16(smem_u32(sm.a[s][rr / BM]) + rt * 128 + ((ch ^ (rt & 7)) << 4), p, src >= 0 ? 16u : 0u);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            if (i >= 1) {   // stage i-1 is complete once at most this stage's group is pending
                asm volatile("cp.async.wait_group 1;" ::: "memory");
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(smem_u32(&sm.full_a[(i - 1) % S]));
            }
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int j = max(0, i - 1); j < i; ++j) mbar_arrive(smem_u32(&sm.full_a[j % S]));
        // ------------------------------------------------------------ epilogue
        const bool ok = __all_sync(0xffffffffu, i == n_iter &&
                                                    mbar_wait(smem_u32(&sm.acc_full), 0, abort_flag, &g_dense_error, kErr));
        if (ok) {
            tc_fence_after();
            // warp w reads the TMEM lane quarter w%4 of tile w/4: its rows are exactly r
            const uint32_t taddr = tmem + mt * BN + ((uint32_t)((warp & 3) * 32) << 16);
            const bool live = r < nrows;
            __nv_bfloat16* dst = out + (row0 + r) * cout + co0;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                float v[32];
                tmem_ld32(taddr + c * 32, v);
                tmem_wait_ld();
                if (live) {
#pragma unroll
                    for (int k = 0; k < 32; ++k) v[k] += __ldg(bias + co0 + c * 32 + k);
#pragma unroll
                    for (int q = 0; q < 4; ++q) *reinterpret_cast<uint4*>(dst + c * 32 + q * 8) = pack8(v + q * 8);
                }
            }
        }
    } else if (warp == GATHER_WARPS) {
        // ------------------------------------------------------------ weight tiles (TMA)
        if (lane == 0) {
            TapWalk tw;
            tw.init(mask, nkc);
            for (int i = 0; i < n_iter; ++i, tw.next()) {
                const int s = i % S;
                if (i >= S && !mbar_wait(smem_u32(&sm.empty[s]), ((i / S) - 1) & 1, abort_flag, &g_dense_error, kErr))
                    break;
                mbar_expect_tx(smem_u32(&sm.full_b[s]), BN * 128);
                tma_load_2d(smem_u32(sm.b[s]), &tmW, tw.kc * BK, tw.tap * cout + co0, smem_u32(&sm.full_b[s]));
            }
        }
    } else {
        // ------------------------------------------------------------ MMA issuer
        // the whole warp runs the loop (every lane waits, the elected lane issues), with the
        // descriptors as per-CTA bases plus stage, tile and k offsets (uniform registers)
        constexpr uint32_t IDESC = make_idesc(BM, BN, false);
        const uint64_t ad0 = make_desc(smem_u32(sm.a[0][0]), 16, 1024, kSw128);
        const uint64_t bd0 = make_desc(smem_u32(sm.b[0]), 16, 1024, kSw128);
        auto wait = [&](uint32_t bar, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, &g_dense_error, kErr));
        };
        bool ok = true;
        for (int i = 0; i < n_iter; ++i) {
            const int s = i % S;
            if (!wait(smem_u32(&sm.full_a[s]), (i / S) & 1) || !wait(smem_u32(&sm.full_b[s]), (i / S) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint64_t bd = bd0 + (uint64_t)(s * (int)(sizeof(sm.b[0]) >> 4));
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                const uint64_t ad = ad0 + (uint64_t)(s * (int)(sizeof(sm.a[0]) >> 4) + t * (int)(sizeof(sm.a[0][0]) >> 4));
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk)
                    tc_mma_elect(tmem + t * BN, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), IDESC,
                                 (i > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit_elect(smem_u32(&sm.empty[s]));
        }
        if (ok) tc_commit_elect(smem_u32(&sm.acc_full));
    }

    tc_fence_before();
    __syncthreads();
    if (warp == GATHER_WARPS + 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

}  // namespace dconv

int dense_conv_error_word(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_dense_error, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    if (clear) {
        int z = 0;
        if (cudaMemcpyToSymbol(g_dense_error, &z, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    }
    return v;
}

}  // namespace vdit

using namespace vdit;

extern "C" int vdit_dense_conv27(const void* f, int64_t n, int32_t cin, int32_t cout, const int32_t* idx,
                                 const void* w, const float* b, void* out, vdit_stream_t stream) {
    using namespace vdit::dconv;
    if (!f || !idx || !w || !b || !out || n < 0 || cin <= 0 || cout <= 0) return VDIT_ERR_ARG;
    if (cin % BK || cout % BN) return VDIT_ERR_UNSUPPORTED;
    if (!aligned16(f) || !aligned16(w) || !aligned16(out)) return VDIT_ERR_ALIGN;
    if (n == 0) return VDIT_OK;
    auto fn = tc::encode_fn();
    if (!fn) return VDIT_ERR_DRIVER;
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)cin, (cuuint64_t)27 * cout};
    cuuint64_t strides[1] = {(cuuint64_t)cin * 2};
    cuuint32_t box[2] = {BK, BN};
    cuuint32_t es[2] = {1, 1};
    if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return VDIT_ERR_DRIVER;
    const size_t sm = sizeof(Smem) + 1024;
    static bool configured = false;
    if (!configured) {
        const cudaError_t e = cudaFuncSetAttribute(dense_conv27_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return VDIT_ERR_LAUNCH;
        }
        configured = true;
    }
    dim3 grid((unsigned)((n + ROWS - 1) / ROWS), (unsigned)(cout / BN));
    dense_conv27_kernel<<<grid, THREADS, sm, static_cast<cudaStream_t>(stream)>>>(
        m, static_cast<const __nv_bfloat16*>(f), n, cin, cout, idx, b, static_cast<__nv_bfloat16*>(out));
    count_launches(1);
    return check_launch();
}
