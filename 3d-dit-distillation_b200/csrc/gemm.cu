// Persistent bf16 GEMM on tcgen05 tensor cores for the block linears:
//   C[M, N] = A[M, K] . W[N, K]^T + bias[N]        (nn.Linear / F.linear layout)
// with epilogues fused where the result feeds a row operation.
//
// CTA pairs (clusters of two, cta_group::2): a pair computes a 256 x 256 output tile
// with 256 x 256 x 16 MMAs issued by the even CTA; each CTA stages its own 128 rows
// of A and its own 128 rows (output columns) of W, so each SM's shared memory feeds
// half the weight tile the pair multiplies.  Pairs walk the tiles t, t + pairs, ...
// (n-major, so the pairs working at one time share weight columns in L2).  Warp roles
// in each CTA:
//   warp 0      TMA producer: A box 64 x 128 and W box 64 x 128 (128-byte swizzle,
//               K-major) per k-step into a 6-stage ring; both CTAs' loads complete on
//               the even CTA's stage barrier, which expects the pair's bytes
//   warp 1      MMA issuer (even CTA, one thread): four MMAs per k-step into one of two
//               TMEM accumulators (2 x 256 fp32 columns = all 512, in both CTAs); its
//               commits arrive on the stage / accumulator barriers of both CTAs
//   warps 2..5  epilogue: warp w drains TMEM lane quarter w % 4 (32 of the CTA's 128
//               rows) while the MMAs of the next tile run into the other accumulator,
//               then arrives on the even CTA's accumulator-free barrier; the qkv epilogue
//               (QK-norm, RoPE, scatter) has eight warps, 2..9, warp w taking head
//               (w - 2) / 4 of the tile's two heads in lane quarter w % 4
// Every mbarrier wait is bounded; a wait that runs out records an error in
// g_gemm_error, raises the CTA abort flag and the CTA skips to its teardown (cluster
// barrier, TMEM always freed).
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "tc.cuh"

namespace vdit {

__device__ int g_gemm_error = 0;

namespace gemm {

using namespace tc;

constexpr int BM = 128;             // rows per CTA (256 per pair)
constexpr int BK = 64;
constexpr int EPI_WARPS = 4;                   // bias epilogue (the qkv epilogue has 8)
constexpr int kErr = 0x474D;   // "GM": a bounded wait of the GEMM kernel ran out

// epilogue kinds
constexpr int EPI_BIAS = 0;   // out = bf16(acc + bias)
constexpr int EPI_QKV = 1;    // self-attention qkv: QK-RMSNorm + 3D RoPE, rows scattered to window order;
                              // a pair tile holds two whole heads (BN = 2 * head_dim, 256 or 192)
constexpr int kQkvTableBytes = 24576;   // EPI_QKV: RoPE cos + sin tables staged in shared memory

// EPI_BIAS: a 6-stage ring (8 for 128-column tiles) and, per epilogue warp, two 32-row x 64-column bf16 boxes stored
// by TMA.  EPI_QKV: a 4-stage ring, the RoPE tables and, per epilogue warp (eight, one head
// each), one buffer of 32 head rows, padded to spread the lanes' stores over the banks; each
// row leaves with its own bulk copy to its scattered output row.
template <int EPI, int BN>
struct __align__(1024) Smem {
    static constexpr int NST = EPI == EPI_QKV ? 4 : BN == 128 ? 8 : 6;
    static constexpr int ROWPAD = BN + 16;                 // a head row: BN / 2 bf16 = BN bytes
    static constexpr int XBYTES =
        EPI == EPI_QKV ? kQkvTableBytes + 8 * 32 * ROWPAD : EPI_WARPS * 2 * 32 * 128;
    uint8_t a[NST][BM * 128];
    uint8_t b[NST][BN / 2 * 128];    // this CTA's half of the weight tile
    uint8_t x[XBYTES];
    uint64_t full[NST], empty[NST], acc_full[2], acc_empty[2];
    uint32_t tmem_slot;
    int abort_flag;
};

struct EpiArgs {
    const __nv_bfloat16* bias;   // [N] or null
    __nv_bfloat16* out;
    int64_t ldo;
    // EPI_QKV only
    const float* q_scale;        // [D] RMSNorm scales of q and k (no +1)
    const float* k_scale;
    const float* cos_t;          // [res, head_dim / 6] RoPE table (staged into shared memory)
    const float* sin_t;
    const int4* coords;          // [M] (b, x, y, z) of each input row
    const int64_t* dst_rows;     // [M] output row of each input row
    int d;                       // heads * 128: columns of each of q, k, v
    int res;
};

// Banded tile order: the pairs walk GM m-tiles x all n-tiles before the next band,
// so the A rows in flight (GM x 256 rows) stay in L2 while every weight column
// passes over them (A of the ffn1 shape, 16384 x 3840, is larger than L2).
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
    constexpr int GM = 8;
    const int g = t / (GM * tiles_n), within = t - g * GM * tiles_n;
    const int gm = min(GM, tiles_m - g * GM);
    tm = g * GM + within % gm;
    tn = within / gm;
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(x), "r"(y)
                 : "memory");
}

// epilogue warps and threads of a kernel kind
template <int EPI>
__host__ __device__ constexpr int epi_warps() { return EPI == EPI_QKV ? 8 : EPI_WARPS; }
template <int EPI>
__host__ __device__ constexpr int threads_of() { return (2 + epi_warps<EPI>()) * 32; }

template <int EPI, int BN>
__global__ void __launch_bounds__(threads_of<EPI>(), 1) gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                          const __grid_constant__ CUtensorMap tmW,
                                                          const __grid_constant__ CUtensorMap tmO, int64_t m, int n,
                                                          int k, const __grid_constant__ EpiArgs ep) {
    extern __shared__ uint8_t raw[];
    constexpr int BNH = BN / 2;                      // weight rows staged per CTA
    constexpr uint32_t kStageBytes = (BM + BNH) * 128;   // per CTA and k-step
    constexpr int kQkvHd = BN / 2;                   // EPI_QKV: head_dim (two heads per tile)
    constexpr int kQkvM = kQkvHd / 6;                // RoPE frequencies per axis (x, y, z)
    using SM = Smem<EPI, BN>;
    constexpr int STAGES = SM::NST;
    SM& sm = *reinterpret_cast<SM*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    volatile int* abort_flag = &sm.abort_flag;
    // a partial last column tile and a partial last k-step read zeros past n and k (the
    // tensor maps' out-of-bounds fill), and the output store is clipped at n columns
    const int tiles_m = (int)((m + 2 * BM - 1) / (2 * BM)), tiles_n = (n + BN - 1) / BN;
    const int ntiles = tiles_m * tiles_n;
    const int nk = (k + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&sm.full[s]), 1);
            mbar_init(smem_u32(&sm.empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&sm.acc_full[b]), 1);
            mbar_init(smem_u32(&sm.acc_empty[b]), 2 * epi_warps<EPI>());
        }
        sm.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmO)) : "memory");
    }
    if (EPI == EPI_QKV) {   // RoPE tables into the staging area (this epilogue stores from registers)
        float* tab = reinterpret_cast<float*>(sm.x);
        const int nt = ep.res * kQkvM;
        for (int i = threadIdx.x; i < nt; i += threads_of<EPI>()) {
            tab[i] = __ldg(ep.cos_t + i);
            tab[nt + i] = __ldg(ep.sin_t + i);
        }
    }
    if (warp == 1) {   // both CTAs of the pair allocate together (same warp, same slot offset)
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&sm.tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    cluster_sync();    // the peer's barriers are initialised before anyone signals them
    tc_fence_after();
    const uint32_t tmem = sm.tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = pair; ok && t < ntiles; t += npairs) {
                int tm, tn;
                tile_coords(t, tiles_m, tiles_n, tm, tn);
                const int arow = tm * 2 * BM + (int)rank * BM, wrow = tn * BN + (int)rank * BNH;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (it >= STAGES &&
                        !mbar_wait(smem_u32(&sm.empty[s]), ((it / STAGES) - 1) & 1, abort_flag, &g_gemm_error, kErr)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full_local = smem_u32(&sm.full[s]);
                    if (leader) mbar_expect_tx(full_local, 2 * kStageBytes);
                    const uint32_t bar = mapa_shared(full_local, 0);
                    tma_load_2d_pair(smem_u32(sm.a[s]), &tmA, kb * BK, arow, bar);
                    tma_load_2d_pair(smem_u32(sm.b[s]), &tmW, kb * BK, wrow, bar);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        // the whole warp runs the loop (every lane waits, the elected lane issues), with the
        // descriptors as per-CTA bases plus stage and k offsets, so they stay in uniform registers
        if (leader) {
            constexpr uint32_t IDESC = make_idesc(2 * BM, BN, false);
            const uint64_t ad0 = make_desc(smem_u32(sm.a[0]), 16, 1024, kSw128);
            const uint64_t bd0 = make_desc(smem_u32(sm.b[0]), 16, 1024, kSw128);
            auto wait = [&](uint32_t bar, uint32_t parity) {
                return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, &g_gemm_error, kErr));
            };
            int it = 0, lt = 0;
            bool ok = true;
            for (int t = pair; ok && t < ntiles; t += npairs, ++lt) {
                const int buf = lt & 1;
                if (lt >= 2 && !wait(smem_u32(&sm.acc_empty[buf]), ((lt >> 1) - 1) & 1)) break;
                tc_fence_after();
                const uint32_t acc = tmem + buf * BN;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (!wait(smem_u32(&sm.full[s]), (it / STAGES) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = ad0 + (uint64_t)(s * (int)(sizeof(sm.a[0]) >> 4));
                    const uint64_t bd = bd0 + (uint64_t)(s * (int)(sizeof(sm.b[0]) >> 4));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        tc_mma_pair_elect(acc, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), IDESC,
                                          (kb > 0 || kk > 0) ? 1u : 0u);
                    tc_commit_pair_elect(smem_u32(&sm.empty[s]), 0x3);
                }
                if (ok) tc_commit_pair_elect(smem_u32(&sm.acc_full[buf]), 0x3);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // Each warp turns 64 columns of its 32 rows at a time into bf16, writes them to one
        // of its two staging boxes (128-byte swizzle: 16-byte chunk j of row r at chunk
        // j ^ (r & 7), so the 32 lanes' stores spread over all banks) and one lane stores
        // the box with TMA; rows past m are clipped by the tensor map.
        const int ew = warp - 2;
        const int quarter = warp & 3;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        int lt = 0, nstore = 0;
        for (int t = pair; t < ntiles; t += npairs, ++lt) {
            const int buf = lt & 1;
            int tm, tn;
            tile_coords(t, tiles_m, tiles_n, tm, tn);
            const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sm.acc_full[buf]), (lt >> 1) & 1, abort_flag,
                                                              &g_gemm_error, kErr));
            if (!ok) break;
            tc_fence_after();
            const int row0 = tm * 2 * BM + (int)rank * BM + quarter * 32;
            const int col0 = tn * BN;
            if (EPI == EPI_BIAS) {
#pragma unroll 1
                for (int c = 0; c < BN / 64; ++c, ++nstore) {
                    float v[64];
                    tmem_ld32(tmem + buf * BN + c * 64 + lane_off, v);
                    tmem_ld32(tmem + buf * BN + c * 64 + 32 + lane_off, v + 32);
                    tmem_wait_ld();
                    if (ep.bias) {
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const int cb = col0 + c * 64 + q * 8;   // n is a multiple of 8
                            if (cb < n) {
                                float bv[8];
                                load8_nc(ep.bias + cb, bv);
#pragma unroll
                                for (int j = 0; j < 8; ++j) v[q * 8 + j] += bv[j];
                            }
                        }
                    }
                    uint8_t* box = sm.x + (ew * 2 + (nstore & 1)) * 32 * 128;
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                    __syncwarp();
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        *reinterpret_cast<uint4*>(box + lane * 128 + ((q ^ (lane & 7)) << 4)) = pack8(v + q * 8);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        // no box starts past m or n (the map clips a box that crosses either)
                        if (row0 < m && col0 + c * 64 < n) tma_store_2d(&tmO, smem_u32(box), col0 + c * 64, row0);
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    }
                }
            }
            if (EPI == EPI_QKV) {
                // one thread per row: the row's two heads of q, k or v; q/k get
                // RoPE3D(bf16(RMSNorm(x)) * scale), exactly as the separate pass computes from
                // the bf16 GEMM output; the row goes to out[dst_rows[row]]
                const int64_t row = (int64_t)row0 + lane;
                const bool live = row < m;
                int64_t orow = 0;
                int tr[3] = {0, 0, 0};
                if (live) {
                    orow = __ldg(ep.dst_rows + row);
                    const int4 c = __ldg(ep.coords + row);
                    tr[0] = min(max(c.y, 0), ep.res - 1) * kQkvM;
                    tr[1] = min(max(c.z, 0), ep.res - 1) * kQkvM;
                    tr[2] = min(max(c.w, 0), ep.res - 1) * kQkvM;
                }
                const float* cs_s = reinterpret_cast<const float*>(sm.x);
                const float* sn_s = cs_s + ep.res * kQkvM;
                {
                    const int hh = ew >> 2;                     // this warp's head of the tile
                    const int col = col0 + hh * kQkvHd;
                    const int section = col / ep.d;                 // 0 q, 1 k, 2 v
                    float x[kQkvHd];
#pragma unroll
                    for (int cc = 0; cc < kQkvHd / 32; ++cc)
                        tmem_ld32(tmem + buf * BN + hh * kQkvHd + cc * 32 + lane_off, x + cc * 32);
                    tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < kQkvHd / 8; ++q) {
                        float bv[8];
                        load8_nc(ep.bias + col + q * 8, bv);
#pragma unroll
                        for (int j = 0; j < 8; ++j) x[q * 8 + j] = bf2f(f2bf(x[q * 8 + j] + bv[j]));
                    }
                    if (section < 2) {
                        float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int e = 0; e < kQkvHd; ++e) ss[e & 3] += x[e] * x[e];
                        const float rr = rsqrtf(((ss[0] + ss[1]) + (ss[2] + ss[3])) / (float)kQkvHd + 1e-6f);
                        const float* sc = (section == 0 ? ep.q_scale : ep.k_scale) + (col - section * ep.d);
#pragma unroll
                        for (int q = 0; q < kQkvHd / 4; ++q) {
                            const float4 s4 = __ldg(reinterpret_cast<const float4*>(sc) + q);
                            x[4 * q + 0] = bf2f(f2bf(x[4 * q + 0] * rr)) * s4.x;
                            x[4 * q + 1] = bf2f(f2bf(x[4 * q + 1] * rr)) * s4.y;
                            x[4 * q + 2] = bf2f(f2bf(x[4 * q + 2] * rr)) * s4.z;
                            x[4 * q + 3] = bf2f(f2bf(x[4 * q + 3] * rr)) * s4.w;
                        }
#pragma unroll
                        for (int g = 0; g < 3; ++g) {
#pragma unroll
                            for (int f = 0; f < kQkvM; ++f) {
                                const int e0 = g * 2 * kQkvM + f, e1 = e0 + kQkvM;
                                const float c = cs_s[tr[g] + f], sn = sn_s[tr[g] + f];
                                const float a = x[e0], b = x[e1];
                                x[e0] = a * c - b * sn;
                                x[e1] = b * c + a * sn;
                            }
                        }
                    }
                    // the row into the warp's buffer (free once the previous tile's copy has been
                    // read), then one bulk copy of its kQkvHd * 2 bytes to the scattered row
                    uint8_t* rb = sm.x + kQkvTableBytes + (ew * 32 + lane) * SM::ROWPAD;
                    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
#pragma unroll
                    for (int q = 0; q < kQkvHd / 8; ++q) *reinterpret_cast<uint4*>(rb + q * 16) = pack8(x + q * 8);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    if (live) {
                        __nv_bfloat16* dst = ep.out + orow * ep.ldo + col;
                        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                                     ::"l"(reinterpret_cast<uint64_t>(dst)), "r"(smem_u32(rb)), "r"(kQkvHd * 2)
                                     : "memory");
                    }
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&sm.acc_empty[buf]), 0));
        }
        if (EPI == EPI_QKV || lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();    // no CTA leaves while its peer's MMAs or arrivals may still touch it
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

bool make_map(CUtensorMap* map, const void* base, int64_t rows, int cols, int64_t ld, int box_rows,
              int box_cols = BK) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            n = 148;
    }
    return n;
}

template <int EPI, int BN>
cudaLaunchConfig_t launch_config(cudaLaunchAttribute* attr, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(threads_of<EPI>());
    cfg.dynamicSmemBytes = sizeof(Smem<EPI, BN>) + 1024;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

// CTA pairs of gemm_kernel<EPI, BN> resident at once on this GPU (queried once; 0 on error).
template <int EPI, int BN>
int max_pairs() {
    static int pairs = 0;
    if (pairs == 0) {
        cudaLaunchAttribute attr[1];
        cudaLaunchConfig_t cfg = launch_config<EPI, BN>(attr, nullptr);
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<EPI, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)cfg.dynamicSmemBytes);
        int p = 0;
        if (e == cudaSuccess) {
            cfg.gridDim = dim3(2 * (num_sms() / 2));
            e = cudaOccupancyMaxActiveClusters(&p, gemm_kernel<EPI, BN>, &cfg);
        }
        if (e != cudaSuccess || p <= 0) {
            record_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidConfiguration);
            return 0;
        }
        pairs = p;
    }
    return pairs;
}

template <int EPI, int BN>
int launch(const CUtensorMap& ma, const CUtensorMap& mw, const CUtensorMap& mo, int64_t m, int n, int k,
           const EpiArgs& ep, cudaStream_t s) {
    const int pairs = max_pairs<EPI, BN>();
    if (pairs <= 0) return VDIT_ERR_LAUNCH;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = launch_config<EPI, BN>(attr, s);
    const int64_t ntiles = ((m + 2 * BM - 1) / (2 * BM)) * ((n + BN - 1) / BN);
    cfg.gridDim = dim3((unsigned)(2 * std::min<int64_t>(ntiles, pairs)));
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_kernel<EPI, BN>, ma, mw, mo, m, n, k, ep);
    if (e != cudaSuccess) {
        record_cuda_error(e);
        return VDIT_ERR_LAUNCH;
    }
    count_launches(1);
    return check_launch();
}

// The pair tile width for an [m, n] output, among 256, 192 and 128 columns that divide n
// (128, with a partial last tile, when none does): the one with the least estimated time,
// rounds of tiles over the resident CTA pairs x the time of one tile.  The mainloop is
// bound by shared-memory bandwidth (MMA operand reads plus TMA fills: 128, 146 and 190
// bytes per clock at the full MMA rate for those widths), so a 192-column tile takes
// 0.75 x 1.17 and a 128-column tile 0.5 x 1.5 of a 256-column tile's time.  The 4101-row
// context linears with n = 1536 come out at 192 (17 x 8 tiles in two rounds of 74 pairs
// instead of 17 x 6 in a second round 38% full); every 16384-row shape keeps 256.
int pick_bn(int64_t m, int n) {
    const int64_t tiles_m = (m + 2 * BM - 1) / (2 * BM);
    const int64_t pairs = std::max(1, num_sms() / 2);
    const int widths[3] = {256, 192, 128};
    const double cost[3] = {1.0, 0.75 * 1.17, 0.5 * 1.5};
    int best = 128;
    double best_t = 1e300;
    for (int i = 0; i < 3; ++i) {
        if (n % widths[i]) continue;
        const int64_t tiles = tiles_m * (n / widths[i]);
        const double t = (double)((tiles + pairs - 1) / pairs) * cost[i];
        if (t < best_t) {
            best_t = t;
            best = widths[i];
        }
    }
    return best;
}

}  // namespace gemm

int gemm_error_word(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    if (clear) {
        int z = 0;
        if (cudaMemcpyToSymbol(g_gemm_error, &z, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    }
    return v;
}

}  // namespace vdit

using namespace vdit;

extern "C" int vdit_linear(const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias, void* out,
                           int64_t ldo, int64_t m, int32_t n, int32_t k, vdit_stream_t stream) {
    using namespace vdit::gemm;
    if (!a || !w || !out || m < 0 || n <= 0 || k <= 0) return VDIT_ERR_ARG;
    if (n % 8 || k % 8) return VDIT_ERR_UNSUPPORTED;
    if (lda < k || ldw < k || ldo < n) return VDIT_ERR_ARG;
    if (!aligned16(a) || !aligned16(w) || !aligned16(out) || (bias && !aligned16(bias)) || lda % 8 || ldw % 8 ||
        ldo % 8)
        return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    if (m > (int64_t)INT32_MAX) return VDIT_ERR_UNSUPPORTED;
    const int bn = pick_bn(m, n);
    CUtensorMap ma, mw, mo;
    if (!make_map(&ma, a, m, k, lda, BM) || !make_map(&mw, w, n, k, ldw, bn / 2) || !make_map(&mo, out, m, n, ldo, 32, 64))
        return VDIT_ERR_DRIVER;
    EpiArgs ep{static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(out), ldo};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (bn == 256) return launch<EPI_BIAS, 256>(ma, mw, mo, m, n, k, ep, s);
    if (bn == 192) return launch<EPI_BIAS, 192>(ma, mw, mo, m, n, k, ep, s);
    return launch<EPI_BIAS, 128>(ma, mw, mo, m, n, k, ep, s);
}

extern "C" int vdit_linear_qkv_rope3d(const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias,
                                      const float* q_scale, const float* k_scale, const float* cos_t,
                                      const float* sin_t, int32_t res, const int32_t* coords,
                                      const int64_t* dst_rows, void* out, int64_t ldo, int64_t m, int32_t heads,
                                      int32_t head_dim, int32_t k, vdit_stream_t stream) {
    using namespace vdit::gemm;
    if (!a || !w || !bias || !q_scale || !k_scale || !cos_t || !sin_t || !coords || !dst_rows || !out || m < 0 ||
        heads <= 0 || k <= 0 || res <= 0)
        return VDIT_ERR_ARG;
    if (head_dim != 128 && head_dim != 96) return VDIT_ERR_UNSUPPORTED;
    const int bn = 2 * head_dim;                 // a pair tile: two whole heads of one section
    const int64_t d = (int64_t)heads * head_dim, n64 = 3 * d;
    if (d % bn || k % BK || n64 > INT32_MAX) return VDIT_ERR_UNSUPPORTED;
    if ((int64_t)res * (head_dim / 6) * 2 * 4 > kQkvTableBytes) return VDIT_ERR_UNSUPPORTED;
    const int n = (int)n64;
    if (lda < k || ldw < k || ldo < n) return VDIT_ERR_ARG;
    if (!aligned16(a) || !aligned16(w) || !aligned16(out) || !aligned16(bias) || !aligned16(q_scale) ||
        !aligned16(k_scale) || !aligned16(coords) || lda % 8 || ldw % 8 || ldo % 8)
        return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    if (m > (int64_t)INT32_MAX) return VDIT_ERR_UNSUPPORTED;
    CUtensorMap ma, mw, mo;
    if (!make_map(&ma, a, m, k, lda, BM) || !make_map(&mw, w, n, k, ldw, bn / 2) || !make_map(&mo, out, m, n, ldo, 32, 64))
        return VDIT_ERR_DRIVER;
    EpiArgs ep{static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(out), ldo, q_scale, k_scale,
               cos_t, sin_t, reinterpret_cast<const int4*>(coords), dst_rows, (int)d, res};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return head_dim == 128 ? launch<EPI_QKV, 256>(ma, mw, mo, m, n, k, ep, s) : launch<EPI_QKV, 192>(ma, mw, mo, m, n, k, ep, s);
}
