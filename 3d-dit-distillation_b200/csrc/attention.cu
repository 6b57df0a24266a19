// Non-causal varlen flash attention on Blackwell tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA computes two 128-query tiles (256 rows) of one head of one segment.
// Warp roles:
//   warp 0      TMA producer: Q (both tiles) once, then K/V tiles of 128 keys into
//               a 2-stage ring
//   warp 1      MMA issuer (one elected thread): S_g = Q_g K^T into TMEM, then
//               O_g += P_g V with P_g read from TMEM (the A operand in tensor memory)
//   warps 2..5  softmax warpgroup of tile 0, warps 6..9 of tile 1: one query row
//               per thread; row max from TMEM, P = exp2(S*scale - m) in fp32 written
//               back to TMEM as bf16 over the S columns, O rescaled in TMEM only when
//               the running max grew by more than 2^8 (exact: the final O/l uses the
//               same reference max); then the epilogue O / l -> bf16 -> global with
//               an optional row scatter.
// While one tile's softmax runs, the tensor core works on the other tile.
// Shared-memory operands use the canonical UMMA layouts: Q/K K-major with 64-byte
// swizzle (TMA boxes of 32 channels), V MN-major with 64-byte swizzle.  Every TMA
// load fills only this CTA's shared memory.  Every mbarrier wait is bounded; a wait that runs
// out records an error in g_device_error, raises a CTA abort flag and the CTA
// skips to its teardown (TMEM is always freed).
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
constexpr int STAGES = 2;
constexpr int THREADS = 320;   // TMA warp, MMA warp, 2 softmax warpgroups
constexpr int MAXSEG = 128;
constexpr int kErrTimeout = 0x4154;   // "AT": a bounded wait of the attention kernel ran out

struct SegInfo {
    int nseg;
    int q0[MAXSEG + 1];
    int k0[MAXSEG + 1];
    int tile0[MAXSEG + 1];
};

// ---------------------------------------------------------------- kernel
// Two 128-row query tiles per CTA (rows q_row0 .. q_row0+255), each with its
// own softmax warpgroup, S/P and O accumulators in TMEM:
//   tile g: S_g (fp32, 128 cols) at col 256g, overwritten in place by P_g
//           (bf16 pairs, 64 cols) once read; O_g at col 256g + 128.
// MMA issue order per key tile j: PV0(j), S0(j+1), PV1(j), S1(j+1), so the
// tensor core computes one tile's products while the other tile's softmax
// runs.  tcgen05 MMAs of one thread execute in issue order, and a commit
// tracks every earlier MMA of that thread, so "S_g(j+1) complete" also means
// "PV_g(j) complete": the softmax group may then rescale O_g and overwrite P_g.
template <int HD>
__global__ void __launch_bounds__(THREADS, 1) attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                              const __grid_constant__ CUtensorMap tmK,
                                                              const __grid_constant__ CUtensorMap tmV,
                                                              __nv_bfloat16* __restrict__ out, int64_t out_stride,
                                                              const int64_t* __restrict__ out_rows,
                                                              const __grid_constant__ SegInfo seg, float scale_log2) {
    constexpr int NCH = HD / 32;                 // 64-byte channel chunks per row
    constexpr int CHUNK = BM * 64;               // bytes of one chunk of a 128-row tile
    constexpr int TILE = NCH * CHUNK;            // bytes of one 128-row Q/K/V tile
    constexpr uint32_t IDESC_QK = make_idesc(BM, BN, false);
    constexpr uint32_t IDESC_PV = make_idesc(BM, HD, true);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                          // [2 tiles]
    uint8_t* sK = sQ + 2 * TILE;                 // [STAGES]
    uint8_t* sV = sK + STAGES * TILE;            // [STAGES]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + STAGES * TILE);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t b_q = smem_u32(&bars[0]);
    auto b_kfull = [&](int s) { return smem_u32(&bars[1 + s]); };
    auto b_kempty = [&](int s) { return smem_u32(&bars[3 + s]); };
    auto b_vfull = [&](int s) { return smem_u32(&bars[5 + s]); };
    auto b_vempty = [&](int s) { return smem_u32(&bars[7 + s]); };
    auto b_sfull = [&](int g) { return smem_u32(&bars[9 + g]); };
    auto b_pfull = [&](int g) { return smem_u32(&bars[11 + g]); };
    auto b_odone = [&](int g) { return smem_u32(&bars[13 + g]); };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.y;
    const int pair = blockIdx.x;
    int s = 0;
    while (s + 1 < seg.nseg && seg.tile0[s + 1] <= pair) ++s;
    const int q_row0 = seg.q0[s] + (pair - seg.tile0[s]) * (2 * BM);
    const int q_rows = min(2 * BM, seg.q0[s + 1] - q_row0);
    const bool has1 = q_rows > BM;                       // CTA-uniform
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
        mbar_init(b_q, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(b_kfull(i), 1);
            mbar_init(b_kempty(i), 1);
            mbar_init(b_vfull(i), 1);
            mbar_init(b_vempty(i), 1);
            mbar_init(b_sfull(i), 1);
            mbar_init(b_pfull(i), 128);
            mbar_init(b_odone(i), 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
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

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            mbar_expect_tx(b_q, (has1 ? 2 : 1) * TILE);
            for (int t = 0; t < (has1 ? 2 : 1); ++t)
                for (int c = 0; c < NCH; ++c)
                    tma_load_3d(smem_u32(sQ + t * TILE + c * CHUNK), &tmQ, c * 32, head, q_row0 + t * BM, b_q);
            // K and V rings with their own barriers: K(j) is free once both S(j) are done,
            // V(j) once both PV(j) are done, so the next K tile can load well before it is needed
            for (int j = 0; j < n_kv; ++j) {
                const int st = j & 1;
                const int krow = k_begin + j * BN;
                if (j >= STAGES &&
                    !mbar_wait(b_kempty(st), ((j - STAGES) >> 1) & 1, abort_flag, &g_device_error, kErrTimeout))
                    break;
                mbar_expect_tx(b_kfull(st), TILE);
                for (int c = 0; c < NCH; ++c)
                    tma_load_3d(smem_u32(sK + st * TILE + c * CHUNK), &tmK, c * 32, head, krow, b_kfull(st));
                if (j >= STAGES &&
                    !mbar_wait(b_vempty(st), ((j - STAGES) >> 1) & 1, abort_flag, &g_device_error, kErrTimeout))
                    break;
                mbar_expect_tx(b_vfull(st), TILE);
                for (int c = 0; c < NCH; ++c)
                    tma_load_3d(smem_u32(sV + st * TILE + c * CHUNK), &tmV, c * 32, head, krow, b_vfull(st));
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const int ntile = has1 ? 2 : 1;
            auto issue_s = [&](int g, int j) {
                const uint32_t qbase = smem_u32(sQ + g * TILE), kbase = smem_u32(sK + (j & 1) * TILE);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = (kk >> 1) * CHUNK + (kk & 1) * 32;
                    tc_mma(tmem + g * 256, make_desc(qbase + off, 16, 512, kSw64),
                           make_desc(kbase + off, 16, 512, kSw64), IDESC_QK, kk > 0 ? 1u : 0u);
                }
            };
            auto issue_pv = [&](int g, int j) {
                const uint32_t vbase = smem_u32(sV + (j & 1) * TILE);
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk) {
                    tc_mma_ts(tmem + g * 256 + 128, tmem + g * 256 + kk * 8, make_desc(vbase + kk * 16 * 64, CHUNK, 512,
                              kSw64), IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
                }
            };
            auto wait = [&](uint32_t bar, uint32_t parity) {
                return mbar_wait(bar, parity, abort_flag, &g_device_error, kErrTimeout);
            };
            bool ok = wait(b_q, 0) && wait(b_kfull(0), 0);
            if (ok) {
                tc_fence_after();
                for (int g = 0; g < ntile; ++g) {
                    issue_s(g, 0);
                    tc_commit(b_sfull(g));
                }
                tc_commit(b_kempty(0));
            }
            for (int j = 0; ok && j < n_kv; ++j) {
                const bool more = j + 1 < n_kv;
                // tile 0: PV0(j) then S0(j+1)
                if (!wait(b_pfull(0), j & 1) || !wait(b_vfull(j & 1), (j >> 1) & 1) ||
                    (more && !wait(b_kfull((j + 1) & 1), ((j + 1) >> 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                issue_pv(0, j);
                if (more) {
                    issue_s(0, j + 1);
                    tc_commit(b_sfull(0));
                } else {
                    tc_commit(b_odone(0));
                }
                // tile 1: PV1(j) then S1(j+1)
                if (ntile > 1) {
                    if (!wait(b_pfull(1), j & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv(1, j);
                }
                tc_commit(b_vempty(j & 1));
                if (ntile > 1) {
                    if (more) {
                        issue_s(1, j + 1);
                        tc_commit(b_sfull(1));
                    } else {
                        tc_commit(b_odone(1));
                    }
                }
                if (more) tc_commit(b_kempty((j + 1) & 1));
            }
        }
    } else {
        // ------------------------------------------------------------ softmax groups
        const int g = (warp - 2) >> 2;                   // query tile of this warpgroup
        const int quarter = warp & 3;                    // TMEM lane quarter this warp may access
        const int row = quarter * 32 + lane;             // row inside the tile
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const uint32_t tS = tmem + g * 256 + lane_off, tO = tS + 128;
        if (g == 0 || has1) {
            float m_run = -INFINITY, l_run = 0.f;
            bool ok = true;
            for (int j = 0; j < n_kv; ++j) {
                // every lane runs each wait, then the warp agrees, so an abort never splits the warp
                ok = __all_sync(0xffffffffu, mbar_wait(b_sfull(g), j & 1, abort_flag, &g_device_error, kErrTimeout));
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
                for (int q = 0; q < 4; ++q) mq[q] = fmaxf(v[q], v[q + 4]);
#pragma unroll
                for (int c = 8; c < BN; c += 8)
#pragma unroll
                    for (int q = 0; q < 4; ++q) mq[q] = fmax3(mq[q], v[c + q], v[c + q + 4]);
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
                // P = exp2(S*scale - m) as bf16 pairs, written over the S columns already read
                float2 lsum[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                  make_float2(0.f, 0.f)};   // independent partial sums
                const float nm = -m_run;
#pragma unroll
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float2 e = ffma2(make_float2(v[c * 32 + i], v[c * 32 + i + 1]), scale_log2, nm);
                        // every eighth pair on the FMA pipe (polynomial exp2), the rest on MUFU, for
                        // which both groups' exponentials contend (1/8 and 1/4 time the same, ~1%
                        // under 1/3); a masked column gives 0 on MUFU and 2^-126 on the polynomial,
                        // and meets a zero-filled V row either way
                        const float2 p = ((i >> 1) % 8 == 7) ? exp2_fma2(e) : make_float2(ex2(e.x), ex2(e.y));
                        lsum[(i >> 1) & 3] = fadd2(lsum[(i >> 1) & 3], p);
                        __nv_bfloat162 bp = __floats2bfloat162_rn(p.x, p.y);
                        pk[i >> 1] = *reinterpret_cast<uint32_t*>(&bp);
                    }
                    tmem_st16(tS + c * 16, pk);
                }
                l_run += (lsum[0].x + lsum[0].y) + (lsum[1].x + lsum[1].y) + (lsum[2].x + lsum[2].y) +
                         (lsum[3].x + lsum[3].y);
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(b_pfull(g));
            }
            // -------------------------------------------------------- epilogue
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(b_odone(g), 0, abort_flag, &g_device_error, kErrTimeout));
            if (ok) {
                tc_fence_after();
                const float inv = 1.f / l_run;
                const int qr = g * BM + row;
                const bool live = qr < q_rows;
                const int64_t orow = live ? (out_rows ? out_rows[q_row0 + qr] : (int64_t)(q_row0 + qr)) : 0;
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
size_t smem_bytes() {
    return 1024 + (size_t)HD * 256 * (2 + 2 * STAGES) + 256;   // tiles + 16 barriers + TMEM slot + abort flag
}

template <int HD>
int launch(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, __nv_bfloat16* out, int64_t out_stride,
           const int64_t* out_rows, const SegInfo& seg, int tiles, int heads, float scale_log2, cudaStream_t s) {
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
    attention_kernel<HD><<<dim3(tiles, heads), THREADS, sm, s>>>(q, k, v, out, out_stride, out_rows, seg, scale_log2);
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
        if (i < nseg) tiles += (cu_q[i + 1] - cu_q[i] + 2 * BM - 1) / (2 * BM);   // 256-row tile pairs
    }
    if (tiles == 0) return VDIT_OK;
    const int64_t q_rows = cu_q[nseg], k_rows = cu_k[nseg];
    CUtensorMap mq, mk, mv;
    if (!make_map(&mq, q, q_rows, heads, hd, q_stride) || !make_map(&mk, k, k_rows, heads, hd, k_stride) ||
        !make_map(&mv, v, k_rows, heads, hd, v_stride))
        return VDIT_ERR_DRIVER;
    const float scale_log2 = scale * 1.4426950408889634f;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
    int rc = hd == 128 ? launch<128>(mq, mk, mv, o, out_stride, out_rows, seg, tiles, heads, scale_log2, s)
                       : launch<96>(mq, mk, mv, o, out_stride, out_rows, seg, tiles, heads, scale_log2, s);
    if (rc != VDIT_OK) return rc;
    count_launches(1);
    return check_launch();
}

namespace vdit {
int dense_conv_error_word(int clear);   // error word of the dense conv kernel (dense_conv.cu)
int dwconv_plan_error_word(int clear);  // error word of the staged depthwise conv (dwconv_plan.cu)
int rowops_error_word(int clear);       // error word of the staged row kernels (rowops.cu)
int gemm_error_word(int clear);         // error word of the tcgen05 GEMM (gemm.cu)
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
    return v != 0 ? v : (d != 0 ? d : (p != 0 ? p : (r != 0 ? r : g)));
}
