// Non-causal varlen flash attention on Blackwell tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA computes one 128-query tile of one head of one segment.  Warp roles:
//   warp 0      TMA producer of K: 128-key tiles into a 4-stage ring
//   warp 1      MMA issuer (converged warp, elected lane): S(j) = Q K(j)^T into one of two
//               score buffers in TMEM, with Q (bf16 pairs) as the A operand in TMEM; then
//               O += P(j) V(j) with P(j) read from TMEM over the score columns of S(j)
//   warps 2..5  softmax warpgroup: one query row per thread; the thread first copies its Q row
//               into TMEM; per key tile: row max from TMEM, P = exp2(S*scale - m) written back
//               to TMEM as bf16 over the S columns, O rescaled in TMEM only when the running
//               max grew by more than 2^8 (exact: the final O/l uses the same reference max),
//               the row sum after the P-ready arrive; then the epilogue O / l -> bf16 -> global
//               with an optional row scatter
//   warp 6      TMA producer of V: 128-key tiles into a 2-stage ring
// MMA issue order: S(0), S(1), then per key tile j: PV(j), S(j+2) into the buffer PV(j) just
// read.  tcgen05 MMAs of one thread execute in issue order, so S(j+2) overwrites P(j) only
// after PV(j) has read it, and the softmax of tile j+1 finds S(j+1) issued a whole tile
// earlier: the tensor core runs while the softmax works, with no second query tile needed.
// Keeping Q in TMEM halves the shared-memory operand traffic of the score MMAs.
// Shared-memory operands use the canonical UMMA layouts: K K-major and V MN-major, both with
// 64-byte swizzle (TMA boxes of 32 channels).  Every TMA load fills only this CTA's shared
// memory.  Every mbarrier wait is bounded; a wait that runs out records an error in
// g_device_error, raises a CTA abort flag and the CTA skips to its teardown (TMEM is always
// freed).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace vdit {

__device__ int g_device_error = 0;

namespace attn {

using namespace tc;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int NS = 2;          // score buffers in TMEM
constexpr int KSTAGES = 4;     // K ring (3 stages measured 0.5% slower, a third V stage 0.5% slower too)
constexpr int VSTAGES = 2;     // V ring
constexpr int POLY8 = 2;       // exp2 pairs (of every 8) on the FMA pipe, the rest on MUFU
constexpr int THREADS = 224;   // K TMA warp, MMA warp, softmax warpgroup, V TMA warp
constexpr int MAXSEG = 128;
constexpr int kErrTimeout = 0x4154;   // "AT": a bounded wait of the attention kernel ran out

struct SegInfo {
    int nseg;
    int q0[MAXSEG + 1];
    int k0[MAXSEG + 1];
    int tile0[MAXSEG + 1];   // first 128-row query tile of each segment
};

// ---------------------------------------------------------------- kernel
// TMEM columns (512 allocated): score buffers b = 0, 1 at 128b (fp32 S, then bf16 P pairs
// over its first 64 columns), O at 256 (HD columns), Q at 256 + HD (HD / 2 columns).
// Barriers, with the phase each wait expects:
//   q          Q copied into TMEM (128 softmax-thread arrivals)
//   kfull/kempty(st), vfull/vempty(st)   the K and V rings (TMA tx / MMA commits)
//   sfull(b)   S(j) complete, j = b mod 2, phase j / 2
//   pfull(b)   P(j) in TMEM (128 arrivals), phase j / 2
//   pvdone(b)  every MMA up to PV(j) complete, phase j / 2 (awaited only before a rescale)
//   odone      the last PV complete
template <int HD>
__global__ void __launch_bounds__(THREADS, 1) attention_kernel(const __grid_constant__ CUtensorMap tmK,
                                                              const __grid_constant__ CUtensorMap tmV,
                                                              const __nv_bfloat16* __restrict__ q, int64_t q_stride,
                                                              __nv_bfloat16* __restrict__ out, int64_t out_stride,
                                                              const int64_t* __restrict__ out_rows,
                                                              const __grid_constant__ SegInfo seg, float scale_log2) {
    constexpr int NCH = HD / 32;                 // 64-byte channel chunks per row
    constexpr int CHUNK = BM * 64;               // bytes of one chunk of a 128-row tile
    constexpr int TILE = NCH * CHUNK;            // bytes of one 128-row K/V tile
    constexpr uint32_t IDESC_QK = make_idesc(BM, BN, false);
    constexpr uint32_t IDESC_PV = make_idesc(BM, HD, true);
    constexpr int OCOL = NS * BN;
    constexpr int QCOL = OCOL + HD;
    static_assert(QCOL + HD / 2 <= 512, "TMEM columns");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sK = smem;                          // [KSTAGES]
    uint8_t* sV = sK + KSTAGES * TILE;           // [VSTAGES]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + VSTAGES * TILE);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t b_q = smem_u32(&bars[0]);
    constexpr int KB = 1, VB = KB + 2 * KSTAGES, SB = VB + 2 * VSTAGES;   // barrier index bases
    static_assert(SB + 3 * NS + 1 <= 24, "barrier slots");
    auto b_kfull = [&](int s) { return smem_u32(&bars[KB + s]); };
    auto b_kempty = [&](int s) { return smem_u32(&bars[KB + KSTAGES + s]); };
    auto b_vfull = [&](int s) { return smem_u32(&bars[VB + s]); };
    auto b_vempty = [&](int s) { return smem_u32(&bars[VB + VSTAGES + s]); };
    auto b_sfull = [&](int b) { return smem_u32(&bars[SB + b]); };
    auto b_pfull = [&](int b) { return smem_u32(&bars[SB + NS + b]); };
    auto b_pvdone = [&](int b) { return smem_u32(&bars[SB + 2 * NS + b]); };
    const uint32_t b_odone = smem_u32(&bars[SB + 3 * NS]);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.y;
    const int tile = blockIdx.x;
    int s = 0;
    while (s + 1 < seg.nseg && seg.tile0[s + 1] <= tile) ++s;
    const int q_row0 = seg.q0[s] + (tile - seg.tile0[s]) * BM;
    const int q_rows = min(BM, seg.q0[s + 1] - q_row0);
    const int k_begin = seg.k0[s];
    const int k_len = seg.k0[s + 1] - k_begin;
    const int n_kv = (k_len + BN - 1) / BN;

    if (n_kv == 0) {   // empty key set: output zeros (uniform for the CTA, before any barrier)
        for (int r = threadIdx.x; r < q_rows; r += THREADS) {
            const int64_t orow = out_rows ? out_rows[q_row0 + r] : (int64_t)(q_row0 + r);
            for (int c = 0; c < HD; ++c) out[orow * out_stride + (int64_t)head * HD + c] = f2bf(0.f);
        }
        return;
    }

    if (threadIdx.x == 0) {
        mbar_init(b_q, 128);
        for (int i = 0; i < KSTAGES; ++i) {
            mbar_init(b_kfull(i), 1);
            mbar_init(b_kempty(i), 1);
        }
        for (int i = 0; i < VSTAGES; ++i) {
            mbar_init(b_vfull(i), 1);
            mbar_init(b_vempty(i), 1);
        }
        for (int b = 0; b < NS; ++b) {
            mbar_init(b_sfull(b), 1);
            mbar_init(b_pfull(b), 128);
            mbar_init(b_pvdone(b), 1);
        }
        mbar_init(b_odone, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmK)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmV)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 || warp == 6) {
        // ------------------------------------------------------------ TMA producers (K: warp 0, V: warp 6)
        // separate rings, so a K tile never waits behind a V slot that a later PV frees
        if (lane == 0) {
            const bool is_k = warp == 0;
            const int nst = is_k ? KSTAGES : VSTAGES;
            const CUtensorMap* map = is_k ? &tmK : &tmV;
            uint8_t* ring = is_k ? sK : sV;
            for (int j = 0; j < n_kv; ++j) {
                const int st = j % nst;
                const uint32_t full = is_k ? b_kfull(st) : b_vfull(st), empty = is_k ? b_kempty(st) : b_vempty(st);
                if (j >= nst && !mbar_wait(empty, ((j - nst) / nst) & 1, abort_flag, &g_device_error, kErrTimeout))
                    break;
                mbar_expect_tx(full, TILE);
                for (int c = 0; c < NCH; ++c)
                    tma_load_3d(smem_u32(ring + st * TILE + c * CHUNK), map, c * 32, head, k_begin + j * BN, full);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // the whole warp runs this loop: every lane waits, the elected lane issues; descriptors
        // are per-CTA bases plus compile-time offsets
        const uint64_t kd0 = make_desc(smem_u32(sK), 16, 512, kSw64);
        const uint64_t vd0 = make_desc(smem_u32(sV), CHUNK, 512, kSw64);
        auto issue_s = [&](int b, int j) {
            const uint64_t kd = kd0 + (uint64_t)((j % KSTAGES) * (TILE >> 4));
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk)
                tc_mma_ts_elect(tmem + b * BN, tmem + QCOL + kk * 8,
                                kd + (uint64_t)(((kk >> 1) * CHUNK + (kk & 1) * 32) >> 4), IDESC_QK, kk > 0 ? 1u : 0u);
        };
        auto issue_pv = [&](int j) {
            const uint64_t vd = vd0 + (uint64_t)((j % VSTAGES) * (TILE >> 4));
            const uint32_t pa = tmem + (j % NS) * BN;
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
                tc_mma_ts_elect(tmem + OCOL, pa + kk * 8, vd + (uint64_t)((kk * 16 * 64) >> 4), IDESC_PV,
                                (j > 0 || kk > 0) ? 1u : 0u);
        };
        auto wait = [&](uint32_t bar, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, &g_device_error, kErrTimeout));
        };
        bool ok = wait(b_q, 0);
        for (int t = 0; ok && t < NS && t < n_kv; ++t) {
            if (!wait(b_kfull(t % KSTAGES), (t / KSTAGES) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            issue_s(t, t);
            tc_commit_elect(b_sfull(t));
            tc_commit_elect(b_kempty(t % KSTAGES));
        }
        for (int j = 0; ok && j < n_kv; ++j) {
            const int b = j % NS;
            if (!wait(b_pfull(b), (j / NS) & 1) || !wait(b_vfull(j % VSTAGES), (j / VSTAGES) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            issue_pv(j);
            tc_commit_elect(b_pvdone(b));
            tc_commit_elect(b_vempty(j % VSTAGES));
            const int jn = j + NS;
            if (jn < n_kv) {
                if (!wait(b_kfull(jn % KSTAGES), (jn / KSTAGES) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                issue_s(b, jn);
                tc_commit_elect(b_sfull(b));
                tc_commit_elect(b_kempty(jn % KSTAGES));
            }
        }
        if (ok) tc_commit_elect(b_odone);
    } else {
        // ------------------------------------------------------------ softmax warpgroup
        const int quarter = warp & 3;                    // TMEM lane quarter this warp may access
        const int row = quarter * 32 + lane;             // row inside the tile
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const uint32_t tO = tmem + lane_off + OCOL;
        {
            // this thread's query row (zeros past the segment) into TMEM as bf16 pairs
            const bool live = row < q_rows;
            const uint4* src =
                reinterpret_cast<const uint4*>(q + (int64_t)(q_row0 + (live ? row : 0)) * q_stride + (int64_t)head * HD);
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                uint32_t w[16];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint4 x = live ? __ldg(src + c * 4 + u) : make_uint4(0, 0, 0, 0);
                    w[4 * u] = x.x;
                    w[4 * u + 1] = x.y;
                    w[4 * u + 2] = x.z;
                    w[4 * u + 3] = x.w;
                }
                tmem_st16(tmem + lane_off + QCOL + c * 16, w);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(b_q);
        }
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            const int b = j % NS;
            const uint32_t tS = tmem + lane_off + b * BN;
            // every lane runs each wait, then the warp agrees, so an abort never splits the warp
            ok = __all_sync(0xffffffffu, mbar_wait(b_sfull(b), (j / NS) & 1, abort_flag, &g_device_error, kErrTimeout));
            if (!ok) break;
            tc_fence_after();
            const int valid = min(BN, k_len - j * BN);
            float v[BN];
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + c * 32, v + c * 32);
            tmem_wait_ld();
            if (valid < BN) {                               // ragged last key tile only
#pragma unroll
                for (int c = 0; c < BN; ++c)
                    if (c >= valid) v[c] = -INFINITY;
            }
            // row max as four independent chains (the reduction is latency-bound otherwise)
            float mq[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) mq[i] = fmaxf(v[i], v[i + 4]);
#pragma unroll
            for (int c = 8; c < BN; c += 8)
#pragma unroll
                for (int i = 0; i < 4; ++i) mq[i] = fmax3(mq[i], v[c + i], v[c + i + 4]);
            const float mt = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
            const float m_new = fmaxf(m_run, mt * scale_log2);
            float alpha = 1.f;
            bool rescale = false;
            if (j == 0) {
                m_run = m_new;
            } else if (m_new > m_run + 8.f) {
                alpha = ex2(m_run - m_new);
                m_run = m_new;
                l_run *= alpha;
                rescale = true;
            }
            if (__any_sync(0xffffffffu, rescale)) {      // warp-uniform TMEM round trip
                // PV(j-1) may still be accumulating into O: wait for it first
                ok = __all_sync(0xffffffffu, mbar_wait(b_pvdone((j - 1) % NS), ((j - 1) / NS) & 1, abort_flag,
                                                       &g_device_error, kErrTimeout));
                if (!ok) break;
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                    float ov[32];
                    tmem_ld32(tO + c * 32, ov);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) ov[i] *= alpha;
                    tmem_st32(tO + c * 32, ov);
                }
            }
            // P = exp2(S*scale - m) as bf16 pairs, written over the S columns already read;
            // the fp32 exponentials stay in v[] for the row sum, which runs after the P-ready
            // arrive so that the tensor core starts PV one sum pass earlier
            const float nm = -m_run;
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float2 e = ffma2(make_float2(v[c * 32 + i], v[c * 32 + i + 1]), scale_log2, nm);
                    // POLY8 of every 8 pairs on the FMA pipe (polynomial exp2), the rest on MUFU;
                    // a masked column gives 0 on MUFU and 2^-126 on the polynomial, and meets a
                    // zero-filled V row either way
                    const float2 p = ((i >> 1) % 8 >= 8 - POLY8) ? exp2_fma2(e) : make_float2(ex2(e.x), ex2(e.y));
                    v[c * 32 + i] = p.x;
                    v[c * 32 + i + 1] = p.y;
                    __nv_bfloat162 bp = __floats2bfloat162_rn(p.x, p.y);
                    pk[i >> 1] = *reinterpret_cast<uint32_t*>(&bp);
                }
                tmem_st16(tS + c * 16, pk);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(b_pfull(b));
            float2 lsum[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};   // independent partial sums
#pragma unroll
            for (int k = 0; k < BN / 2; ++k) lsum[k & 3] = fadd2(lsum[k & 3], make_float2(v[2 * k], v[2 * k + 1]));
            l_run += (lsum[0].x + lsum[0].y) + (lsum[1].x + lsum[1].y) + (lsum[2].x + lsum[2].y) +
                     (lsum[3].x + lsum[3].y);
        }
        // ------------------------------------------------------------ epilogue
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(b_odone, 0, abort_flag, &g_device_error, kErrTimeout));
        if (ok) {
            tc_fence_after();
            const float inv = 1.f / l_run;
            const bool live = row < q_rows;
            const int64_t orow = live ? (out_rows ? out_rows[q_row0 + row] : (int64_t)(q_row0 + row)) : 0;
            __nv_bfloat16* dst = out + orow * out_stride + (int64_t)head * HD;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                float ov[32];
                tmem_ld32(tO + c * 32, ov);
                tmem_wait_ld();
                if (live) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) ov[i] *= inv;
#pragma unroll
                    for (int v = 0; v < 4; ++v) *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = pack8(ov + v * 8);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

// ---------------------------------------------------------------- host side
}  // namespace attn

namespace tc {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}
}  // namespace tc

namespace attn {

bool make_map(CUtensorMap* m, const void* base, int64_t rows, int heads, int hd, int64_t row_stride) {
    auto fn = tc::encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)heads, (cuuint64_t)rows};
    cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)row_stride * 2};
    cuuint32_t box[3] = {32, 1, (cuuint32_t)BM};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int HD>
size_t smem_bytes() {   // alignment slack + K and V rings + 24 barriers + TMEM slot + abort flag
    return 1024 + (size_t)HD * 256 * (KSTAGES + VSTAGES) + 256;
}

template <int HD>
int launch(const CUtensorMap& k, const CUtensorMap& v, const __nv_bfloat16* q, int64_t q_stride, __nv_bfloat16* out,
           int64_t out_stride, const int64_t* out_rows, const SegInfo& seg, int tiles, int heads, float scale_log2,
           cudaStream_t s) {
    static bool configured = false;
    const size_t sm = smem_bytes<HD>();
    if (!configured) {
        const cudaError_t e = cudaFuncSetAttribute(attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return VDIT_ERR_LAUNCH;
        }
        configured = true;
    }
    attention_kernel<HD><<<dim3(tiles, heads), THREADS, sm, s>>>(k, v, q, q_stride, out, out_stride, out_rows, seg,
                                                                 scale_log2);
    return VDIT_OK;
}

}  // namespace attn
}  // namespace vdit

using namespace vdit;

extern "C" int vdit_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                              int64_t v_stride, void* out, int64_t out_stride, const int64_t* out_rows,
                              const int32_t* cu_q, const int32_t* cu_k, int32_t nseg, int32_t heads, int32_t hd,
                              float scale, vdit_stream_t stream) {
    using namespace vdit::attn;
    if (!q || !k || !v || !out || !cu_q || !cu_k || nseg < 1 || heads < 1) return VDIT_ERR_ARG;
    if (nseg > MAXSEG) return VDIT_ERR_UNSUPPORTED;
    if (hd != 96 && hd != 128) return VDIT_ERR_UNSUPPORTED;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || q_stride % 8 || k_stride % 8 ||
        v_stride % 8 || out_stride % 8)
        return VDIT_ERR_ALIGN;
    if (q_stride < (int64_t)heads * hd || k_stride < (int64_t)heads * hd || v_stride < (int64_t)heads * hd ||
        out_stride < (int64_t)heads * hd)
        return VDIT_ERR_ARG;
    SegInfo seg;
    memset(&seg, 0, sizeof(seg));
    seg.nseg = nseg;
    int tiles = 0;
    for (int i = 0; i <= nseg; ++i) {
        if (cu_q[i] < 0 || cu_k[i] < 0) return VDIT_ERR_ARG;
        if (i > 0 && (cu_q[i] < cu_q[i - 1] || cu_k[i] < cu_k[i - 1])) return VDIT_ERR_ARG;
        seg.q0[i] = cu_q[i];
        seg.k0[i] = cu_k[i];
        seg.tile0[i] = tiles;
        if (i < nseg) tiles += (cu_q[i + 1] - cu_q[i] + BM - 1) / BM;   // 128-row query tiles
    }
    if (tiles == 0) return VDIT_OK;
    const int64_t k_rows = cu_k[nseg];
    CUtensorMap mk, mv;
    if (!make_map(&mk, k, k_rows, heads, hd, k_stride) || !make_map(&mv, v, k_rows, heads, hd, v_stride))
        return VDIT_ERR_DRIVER;
    const float scale_log2 = scale * 1.4426950408889634f;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
    const __nv_bfloat16* qb = static_cast<const __nv_bfloat16*>(q);
    int rc = hd == 128 ? launch<128>(mk, mv, qb, q_stride, o, out_stride, out_rows, seg, tiles, heads, scale_log2, s)
                       : launch<96>(mk, mv, qb, q_stride, o, out_stride, out_rows, seg, tiles, heads, scale_log2, s);
    if (rc != VDIT_OK) return rc;
    count_launches(1);
    return check_launch();
}

namespace vdit {
int dense_conv_error_word(int clear);   // error word of the dense conv kernel (dense_conv.cu)
int dwconv_plan_error_word(int clear);  // error word of the staged depthwise conv (dwconv_plan.cu)
int rowops_error_word(int clear);       // error word of the staged row kernels (rowops.cu)
int gemm_error_word(int clear);         // error word of the tcgen05 GEMM (gemm.cu)
int unpatch_error_word(int clear);      // error word of the unpatchify projection (unpatchify.cu)
int patchify_error_word(int clear);     // error word of the tensor-core patchify (patchify.cu)
}

extern "C" int vdit_device_error(int clear) {
    int v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return VDIT_ERR_LAUNCH;
    if (cudaMemcpyFromSymbol(&v, vdit::g_device_error, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    if (clear) {
        int z = 0;
        if (cudaMemcpyToSymbol(vdit::g_device_error, &z, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    }
    const int d = vdit::dense_conv_error_word(clear);
    if (d < 0) return d;
    const int p = vdit::dwconv_plan_error_word(clear);
    if (p < 0) return p;
    const int r = vdit::rowops_error_word(clear);
    if (r < 0) return r;
    const int g = vdit::gemm_error_word(clear);
    if (g < 0) return g;
    const int u = vdit::unpatch_error_word(clear);
    if (u < 0) return u;
    const int t = vdit::patchify_error_word(clear);
    if (t < 0) return t;
    for (int w : {v, d, p, r, g, u, t})
        if (w != 0) return w;
    return 0;
}
