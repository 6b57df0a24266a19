// Depthwise 27-tap sparse conv + SwiGLU with neighbour rows staged in shared
// memory ("planned" variant of dwconv27 with fuse_swiglu).
//
// The gather form reads every present neighbour of every output row from L2:
// 13.4 taps per row on a surface-like voxel set, i.e. about 13x the feature
// bytes cross the L2->SM path while DRAM sees the input once.  Here the rows
// are cut into blocks of 128 consecutive voxels along the Hilbert curve (a
// compact surface patch); the union of a block's neighbours is ~1.8x its size
// on a surface.  A plan built once per voxel set (the conv indices do not
// change across layers or solver steps) lists, per block, the union ("slots")
// and, per group of 4 output rows, the union of the rows' taps as a compact
// list with the slot of each (row, tap).  Rows are grouped greedily so that a
// group's union stays small (18.3 taps for 13.4 present per row on the shell
// workload).  The conv kernel copies a block's slots x one 64-channel tile of
// a and gate into shared memory once and computes all 128 rows from there.
//
// Layout: the packed hidden h' [n, c] is pair-interleaved -- columns
// 4k..4k+3 hold (a[2k], a[2k+1], gate[2k], gate[2k+1]) -- and so are the conv
// weights w' [27, c] and bias b' [c]; the output is silu(gate) * a in natural
// channel order [n, c/2].  The runner obtains this layout for free by
// permuting the rows of the up-projection that produces h.  A lane then reads
// its 2 a + 2 gate values with one 8-byte load and its 4 weights with one
// 16-byte load, and one TMA row copy covers a whole tile.
//
// Mapping: a persistent CTA (one per SM) walks work units (tile, block) in
// tile-major order.  One producer warp stages unit u+1 while 16 compute warps
// work on unit u: TMA tile::gather4 copies four slot rows x 128 columns per
// instruction, bulk copies bring the group table and (when the tile changes)
// the tile's weights, and an mbarrier pair per stage hands the buffer over
// (waits are bounded; a timeout sets the device error word).  A warp computes
// one group of 4 rows at a time, lane l owning output channels (2l, 2l+1) of
// the tile; a row without one of the group's taps reads a zero row.
// Accumulation order (bias, then taps in increasing index) and fp32 FMAs match
// the gather kernel, so results are bit-identical to it on the de-interleaved
// inputs.  Blocks whose union exceeds the slot capacity (dense volumes, or a
// row order that is not a space-filling curve) keep global row indices in the
// plan and are computed from global memory.
#include "common.cuh"
#include "tc.cuh"

namespace vdit {
namespace {

constexpr int kPlanRows = 128;                 // output rows per block
constexpr int kGroupRows = 4;                  // rows per group (one warp step)
constexpr int kGroups = kPlanRows / kGroupRows;
constexpr int kSlotCap = 320;                  // staged union rows per block
constexpr int kCand = kPlanRows * 27;          // neighbour candidates per block
constexpr int kSortN = 4096;                   // power of two >= kCand
constexpr int kTileCh = 64;                    // output channels per tile
constexpr int kTileCols = 2 * kTileCh;         // h' columns per tile (a + gate)
constexpr int kSlotBytes = kTileCols * 2;      // bf16
constexpr int kWarps = 16;                     // compute warps (+1 producer warp)

struct __align__(16) Group {
    int32_t rows[kGroupRows];      // output rows (-1: padding)
    int32_t ntaps;                 // taps in the group's union
    int32_t pad[3];
    uint8_t taps[32];              // the union's tap indices, increasing
    int4 slots[27];                // per union tap: byte offset of each row's staged slot
                                   // (the zero row if the row lacks the tap), or on
                                   // overflow its global row (-1 if absent)
};
static_assert(sizeof(Group) == 496, "group layout");

struct __align__(16) BlockHdr {
    int32_t n_slots;               // union size
    int32_t overflow;              // 1: slots hold global rows, compute from global memory
    int32_t pad[2];
};

constexpr size_t kHdrBytes = sizeof(BlockHdr);
constexpr size_t kSlotListBytes = (size_t)kSlotCap * 4;
constexpr size_t kGroupTabBytes = (size_t)kGroups * sizeof(Group);
constexpr size_t kBlockPlanBytes = kHdrBytes + kSlotListBytes + kGroupTabBytes;

// Stage layout: slot s at s*256 (a quad of four slots is one TMA gather4),
// the zero row after the last slot, then the block's group table.  After the
// two stages: two weight buffers (indexed by tile parity), each 27 taps + bias
// x 128 fp32 columns; then barriers and flags.
constexpr int kZeroOff = kSlotCap * kSlotBytes;
constexpr int kStageFeat = kZeroOff + kSlotBytes;
constexpr int kStageBytes = kStageFeat + (int)kGroupTabBytes;
constexpr int kWRowBytes = kTileCols * 4;
constexpr int kWBytes = 28 * kWRowBytes;
constexpr int kWOff = 2 * kStageBytes;
constexpr int kBarOff = kWOff + 2 * kWBytes;
constexpr int kSmemBytes = kBarOff + 64;
static_assert(kStageFeat % 128 == 0 && kStageBytes % 128 == 0 && kWOff % 128 == 0, "stage alignment");
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");

struct PlanView {
    BlockHdr* hdr;
    int32_t* slot_rows;            // [blocks][kSlotCap]: global row of slot s (row 0 past the union)
    Group* groups;                 // [blocks][kGroups]
};

__host__ __device__ inline PlanView plan_view(void* plan, int64_t blocks) {
    char* p = static_cast<char*>(plan);
    PlanView v;
    v.hdr = reinterpret_cast<BlockHdr*>(p);
    v.slot_rows = reinterpret_cast<int32_t*>(p + blocks * kHdrBytes);
    v.groups = reinterpret_cast<Group*>(p + blocks * (kHdrBytes + kSlotListBytes));
    return v;
}

// ---------------------------------------------------------------- plan build
// One CTA per block: gather the 128x27 neighbour indices, sort them (bitonic,
// shared memory), keep the distinct ones as slots, map every (row, tap) to its
// slot by binary search, group the rows greedily (seed: the remaining row with
// the most taps; then three times the row that grows the union least; padding
// rows last), improve the groups by pairwise row swaps, and write the group records.
__global__ void __launch_bounds__(512) dwconv_plan_kernel(const int32_t* __restrict__ idx,
                                                          const int64_t* __restrict__ order, int64_t n,
                                                          int64_t blocks, void* plan) {
    __shared__ int32_t nb[kCand];
    __shared__ int32_t cand[kSortN];
    __shared__ int32_t warp_tot[16];
    __shared__ int32_t rowid[kPlanRows];
    __shared__ uint32_t mask[kPlanRows];
    __shared__ int32_t grp_row[kGroups][kGroupRows];   // positions within the block
    __shared__ uint32_t grp_mask[kGroups];
    __shared__ int32_t n_uniq;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t blk = blockIdx.x;
    PlanView pv = plan_view(plan, blocks);

    if (tid < kPlanRows) {
        const int64_t i = blk * kPlanRows + tid;
        rowid[tid] = i < n ? (int32_t)__ldg(order + i) : -1;
    }
    __syncthreads();
    for (int k = tid; k < kCand; k += blockDim.x) {
        const int r = rowid[k / 27];
        nb[k] = r >= 0 ? __ldg(idx + (int64_t)r * 27 + k % 27) : -1;
    }
    __syncthreads();
    for (int k = tid; k < kSortN; k += blockDim.x) cand[k] = (k < kCand && nb[k] >= 0) ? nb[k] : INT32_MAX;
    if (tid < kPlanRows) {
        uint32_t m = 0;
        for (int d = 0; d < 27; ++d) m |= (nb[tid * 27 + d] >= 0 ? 1u : 0u) << d;
        mask[tid] = m;
    }
    __syncthreads();
    if (warp == 0) {
        // greedy grouping; lane l holds rows l, l+32, l+64, l+96
        constexpr int kPerLane = kPlanRows / 32;
        uint32_t mk[kPerLane];
        bool real[kPerLane], left[kPerLane];
#pragma unroll
        for (int j = 0; j < kPerLane; ++j) {
            mk[j] = mask[lane + 32 * j];
            real[j] = rowid[lane + 32 * j] >= 0;
            left[j] = true;
        }
        for (int g = 0; g < kGroups; ++g) {
            uint32_t u = 0;
            for (int q = 0; q < kGroupRows; ++q) {
                // smallest key wins: real rows before padding; seed = most taps, then
                // the least union growth; ties to the lowest position
                uint32_t best = 0xffffffffu;
#pragma unroll
                for (int j = 0; j < kPerLane; ++j) {
                    if (!left[j]) continue;
                    const uint32_t r = lane + 32 * j;
                    const uint32_t score = q == 0 ? 27u - __popc(mk[j]) : __popc(u | mk[j]);
                    const uint32_t key = ((real[j] ? 0u : 1u) << 20) | (score << 8) | r;
                    best = min(best, key);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
                const int r = (int)(best & 0xff);
#pragma unroll
                for (int j = 0; j < kPerLane; ++j)
                    if (r == lane + 32 * j) left[j] = false;
                u |= mask[r];
                if (lane == 0) grp_row[g][q] = r;
            }
            if (lane == 0) grp_mask[g] = u;
        }
        __syncwarp();
        // two sweeps of pairwise swaps between groups: for every pair of groups the 16 row
        // swaps are scored in parallel (lane = 4i + j swaps row i of a with row j of b) and
        // the one that shrinks the two unions most is applied (on the shell test sets this
        // takes the mean union from 18.4 to 17.7 taps per row)
        for (int sweep = 0; sweep < 2; ++sweep) {
            for (int a = 0; a < kGroups; ++a) {
                for (int b = a + 1; b < kGroups; ++b) {
                    uint32_t key = 0;
                    if (lane < 16) {
                        const int i = lane >> 2, j = lane & 3;
                        uint32_t ua = mask[grp_row[b][j]], ub = mask[grp_row[a][i]];
#pragma unroll
                        for (int q = 0; q < kGroupRows; ++q) {
                            if (q != i) ua |= mask[grp_row[a][q]];
                            if (q != j) ub |= mask[grp_row[b][q]];
                        }
                        const int gain = __popc(grp_mask[a]) + __popc(grp_mask[b]) - __popc(ua) - __popc(ub);
                        if (gain > 0) key = ((uint32_t)gain << 8) | (uint32_t)(31 - lane);
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
                    if (key != 0 && lane == 0) {
                        const int l = 31 - (int)(key & 0xff), i = l >> 2, j = l & 3;
                        const int ra = grp_row[a][i];
                        grp_row[a][i] = grp_row[b][j];
                        grp_row[b][j] = ra;
                        uint32_t ua = 0, ub = 0;
                        for (int q = 0; q < kGroupRows; ++q) {
                            ua |= mask[grp_row[a][q]];
                            ub |= mask[grp_row[b][q]];
                        }
                        grp_mask[a] = ua;
                        grp_mask[b] = ub;
                    }
                    __syncwarp();
                }
            }
        }
    }
    // bitonic sort of the candidates, ascending
    for (int size = 2; size <= kSortN; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = tid; t < kSortN / 2; t += blockDim.x) {
                const int lo = 2 * t - (t & (stride - 1));
                const int hi = lo + stride;
                const bool up = (lo & size) == 0;
                const int32_t a = cand[lo], c = cand[hi];
                if ((a > c) == up) {
                    cand[lo] = c;
                    cand[hi] = a;
                }
            }
            __syncthreads();
        }
    }
    // distinct values -> cand[0, U)   (each thread owns 8 consecutive entries)
    constexpr int kPer = kSortN / 512;
    int32_t v[kPer];
    bool first[kPer];
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int k = tid * kPer + j;
        v[j] = cand[k];
        first[j] = v[j] != INT32_MAX && (k == 0 || cand[k - 1] != v[j]);
        cnt += first[j];
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < warp; ++w) base += warp_tot[w];
    if (tid == blockDim.x - 1) n_uniq = base + incl;
    int pos = base + incl - cnt;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
        if (first[j]) cand[pos++] = v[j];
    __syncthreads();
    const int U = n_uniq;
    const bool overflow = U > kSlotCap;
    // (row, tap) -> byte offset of slot p (p = position among the distinct rows),
    // the zero row for an absent tap; on overflow the global row itself (-1 when absent)
    for (int k = tid; k < kCand; k += blockDim.x) {
        const int32_t x = nb[k];
        int32_t s;
        if (overflow) {
            s = x;
        } else if (x < 0) {
            s = kZeroOff;
        } else {
            int lo = 0, hi = U;
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (cand[mid] < x) lo = mid + 1; else hi = mid;
            }
            s = lo * kSlotBytes;
        }
        nb[k] = s;
    }
    __syncthreads();
    if (tid == 0) {
        BlockHdr h;
        h.n_slots = overflow ? 0 : U;
        h.overflow = overflow ? 1 : 0;
        h.pad[0] = h.pad[1] = 0;
        pv.hdr[blk] = h;
    }
    for (int s = tid; s < kSlotCap; s += blockDim.x) pv.slot_rows[blk * kSlotCap + s] = (!overflow && s < U) ? cand[s] : 0;
    Group* g = pv.groups + blk * kGroups;
    if (tid < kGroups) {
        const uint32_t m = grp_mask[tid];
        for (int q = 0; q < kGroupRows; ++q) g[tid].rows[q] = rowid[grp_row[tid][q]];
        g[tid].ntaps = __popc(m);
        g[tid].pad[0] = g[tid].pad[1] = g[tid].pad[2] = 0;
        int i = 0;
        for (int d = 0; d < 27; ++d)
            if (m & (1u << d)) g[tid].taps[i++] = (uint8_t)d;
        for (; i < 32; ++i) g[tid].taps[i] = 0;
    }
    for (int k = tid; k < kGroups * 27 * kGroupRows; k += blockDim.x) {
        const int gi = k / (27 * kGroupRows), i = (k / kGroupRows) % 27, q = k % kGroupRows;
        const uint32_t m = grp_mask[gi];
        int32_t s = overflow ? -1 : kZeroOff;
        if (i < __popc(m)) {
            const int d = (int)__fns(m, 0, i + 1);      // the i-th tap of the union
            const int r = grp_row[gi][q];
            if (rowid[r] >= 0) s = nb[r * 27 + d];
        }
        reinterpret_cast<int32_t*>(&g[gi].slots[i])[q] = s;
    }
}

// ---------------------------------------------------------------- conv
__device__ int g_dwplan_error = 0;
constexpr int kErrTimeout = 3;

// d.x += bf16(x.lo) * bf16(w.lo), d.y += bf16(x.hi) * bf16(w.hi): fp32 FMAs with operands read
// straight from packed bf16 registers (fma.rn.f32.bf16: exact inputs, one rounding), which
// saves the unpack of the features when the weights are bf16 values too
__device__ __forceinline__ void fma_bf2(float2& d, uint32_t x, uint32_t w) {
    asm("{.reg .b16 x0, x1, w0, w1;\n\t"
        "mov.b32 {x0, x1}, %2;\n\t"
        "mov.b32 {w0, w1}, %3;\n\t"
        "fma.rn.f32.bf16 %0, x0, w0, %0;\n\t"
        "fma.rn.f32.bf16 %1, x1, w1, %1;\n\t}"
        : "+f"(d.x), "+f"(d.y) : "r"(x), "r"(w));
}

__device__ __forceinline__ float2 unpack_bf2(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// four rows x 128 bf16 columns of h' -> 1024 contiguous bytes of shared memory
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, int col, int4 rows, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(col), "r"(rows.x), "r"(rows.y), "r"(rows.z),
          "r"(rows.w), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Accumulates one group of 4 rows over its union taps, two taps per iteration
// (both taps' loads issued before their FMAs).  BF16W: the weights hold bf16 values, so each
// tap's four weights are packed to bf16 (exactly) and the FMAs take bf16 operands directly;
// the products and sums are the same fp32 operations either way.
template <bool GLOBAL, bool BF16W>
__device__ __forceinline__ void accumulate_group(const Group* grp, const char* feat, const char* wb, int lane,
                                                 const __nv_bfloat16* __restrict__ hcol, int c,
                                                 float2 (&acc_a)[kGroupRows], float2 (&acc_g)[kGroupRows]) {
    const int nt = grp->ntaps;
    const char* fl = feat + lane * 8;
    const char* wl = wb + lane * 16;
    auto load_tap = [&](int i, uint2 (&v)[kGroupRows], float4& wv) {
        const int4 sl = grp->slots[i];
        const int s[kGroupRows] = {sl.x, sl.y, sl.z, sl.w};
#pragma unroll
        for (int q = 0; q < kGroupRows; ++q) {
            if (GLOBAL) {
                const bool ok = s[q] >= 0;
                const uint2* p = reinterpret_cast<const uint2*>(hcol + (int64_t)(ok ? s[q] : 0) * c);
                v[q] = ok ? __ldg(p) : make_uint2(0u, 0u);
            } else {
                v[q] = *reinterpret_cast<const uint2*>(fl + s[q]);
            }
        }
        wv = *reinterpret_cast<const float4*>(wl + grp->taps[i] * kWRowBytes);
    };
    auto fma_tap = [&](const uint2 (&v)[kGroupRows], const float4& wv) {
        if (BF16W) {
            __nv_bfloat162 wa2 = __floats2bfloat162_rn(wv.x, wv.y), wg2 = __floats2bfloat162_rn(wv.z, wv.w);
            const uint32_t wa = *reinterpret_cast<uint32_t*>(&wa2), wg = *reinterpret_cast<uint32_t*>(&wg2);
#pragma unroll
            for (int q = 0; q < kGroupRows; ++q) {
                fma_bf2(acc_a[q], v[q].x, wa);
                fma_bf2(acc_g[q], v[q].y, wg);
            }
        } else {
            const float2 wa = make_float2(wv.x, wv.y), wg = make_float2(wv.z, wv.w);
#pragma unroll
            for (int q = 0; q < kGroupRows; ++q) {
                acc_a[q] = tc::ffma2v(unpack_bf2(v[q].x), wa, acc_a[q]);
                acc_g[q] = tc::ffma2v(unpack_bf2(v[q].y), wg, acc_g[q]);
            }
        }
    };
    int i = 0;
    for (; i + 1 < nt; i += 2) {
        uint2 v0[kGroupRows], v1[kGroupRows];
        float4 w0, w1;
        load_tap(i, v0, w0);
        load_tap(i + 1, v1, w1);
        fma_tap(v0, w0);
        fma_tap(v1, w1);
    }
    if (i < nt) {
        uint2 v0[kGroupRows];
        float4 w0;
        load_tap(i, v0, w0);
        fma_tap(v0, w0);
    }
}

// Warps 0..15 compute; warp 16 stages work units into a two-slot ring
// (full: TMA bytes landed; empty: the compute warps are done with it).
template <bool BF16W>
__global__ void __launch_bounds__((kWarps + 1) * 32, 1) dwconv_planned_kernel(
        const __grid_constant__ CUtensorMap hmap, const __nv_bfloat16* __restrict__ h, int c,
        const void* __restrict__ plan, int64_t blocks, const float* __restrict__ w, const float* __restrict__ b,
        __nv_bfloat16* __restrict__ out) {
    using namespace tc;
    extern __shared__ __align__(1024) char smem[];
    const PlanView pv = plan_view(const_cast<void*>(plan), blocks);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int half = c / 2;
    const int64_t tiles = c / kTileCols;
    const int64_t units = blocks * tiles;
    const int64_t u0 = units * blockIdx.x / gridDim.x;
    const int64_t u1 = units * (blockIdx.x + 1) / gridDim.x;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + kBarOff;            // full[0], full[1], empty[0], empty[1]
    int* info = reinterpret_cast<int*>(smem + kBarOff + 32);   // per stage: overflow flag
    volatile int* abort_flag = info + 2;
    auto full = [&](int st) { return bars + 8 * st; };
    auto empty = [&](int st) { return bars + 16 + 8 * st; };

    if (tid == 0) {
        for (int st = 0; st < 2; ++st) {
            mbar_init(full(st), 1);
            mbar_init(empty(st), kWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // the zero rows of both stages (absent taps read them)
    for (int k = tid; k < 2 * kSlotBytes / 16; k += blockDim.x) {
        constexpr int per = kSlotBytes / 16;
        reinterpret_cast<uint4*>(smem + (k / per) * kStageBytes + kZeroOff)[k % per] = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();

    if (warp == kWarps) {
        // ---------------- producer
        int64_t issued = 0, w_tile = -1;
        for (int64_t u = u0; u < u1; ++u, ++issued) {
            const int st = (int)(issued & 1);
            const uint32_t k = (uint32_t)(issued >> 1);
            // stage st was last used by unit issued-2; weight buffer tile&1 last by a unit
            // of tile-2, which precedes it, so this wait frees both
            if (issued >= 2 && !__all_sync(0xffffffffu, mbar_wait(empty(st), (k - 1) & 1, abort_flag,
                                                                   &g_dwplan_error, kErrTimeout)))
                break;
            const int64_t tile = u / blocks, blk = u % blocks;
            const BlockHdr hd = pv.hdr[blk];
            const int nq = hd.overflow ? 0 : (hd.n_slots + 3) / 4;
            const bool new_w = tile != w_tile;
            const uint32_t dst = sbase + st * kStageBytes;
            const int col = (int)(tile * kTileCols);
            if (lane == 0) {
                info[st] = hd.overflow;
                mbar_expect_tx(full(st), (uint32_t)kGroupTabBytes + (uint32_t)nq * 4 * kSlotBytes +
                                             (new_w ? (uint32_t)kWBytes : 0u));
                bulk_copy(dst + kStageFeat, pv.groups + blk * kGroups, (uint32_t)kGroupTabBytes, full(st));
            }
            __syncwarp();
            if (new_w && lane < 28) {
                const uint32_t wdst = sbase + kWOff + (uint32_t)(tile & 1) * kWBytes + lane * kWRowBytes;
                const float* src = lane < 27 ? w + (int64_t)lane * c : b;
                bulk_copy(wdst, src + col, kWRowBytes, full(st));
            }
            w_tile = tile;
            const int4* rows4 = reinterpret_cast<const int4*>(pv.slot_rows + blk * kSlotCap);
            for (int q = lane; q < nq; q += 32)
                tma_gather4(dst + q * 4 * kSlotBytes, &hmap, col, __ldg(rows4 + q), full(st));
        }
        // nothing may still be landing in shared memory when the CTA exits
        if (lane == 0)
            for (int64_t j = (issued > 2 ? issued - 2 : 0); j < issued; ++j)
                mbar_wait(full((int)(j & 1)), (uint32_t)(j >> 1) & 1, abort_flag, &g_dwplan_error, kErrTimeout);
        return;
    }

    // ---------------- consumers
    int64_t used = 0;
    for (int64_t u = u0; u < u1; ++u, ++used) {
        const int st = (int)(used & 1);
        if (!__all_sync(0xffffffffu, mbar_wait(full(st), (uint32_t)(used >> 1) & 1, abort_flag, &g_dwplan_error,
                                               kErrTimeout)))
            break;
        const int64_t tile = u / blocks;
        const bool overflow = info[st] != 0;
        const char* feat = smem + st * kStageBytes;
        const char* wb = smem + kWOff + (tile & 1) * kWBytes;
        const float4 bias = *reinterpret_cast<const float4*>(wb + 27 * kWRowBytes + lane * 16);
        const __nv_bfloat16* hcol = h + tile * kTileCols + lane * 4;
        __nv_bfloat16* ocol = out + tile * kTileCh + lane * 2;
        for (int gi = warp; gi < kGroups; gi += kWarps) {
            const Group* grp = reinterpret_cast<const Group*>(feat + kStageFeat) + gi;
            const int4 rows4 = *reinterpret_cast<const int4*>(grp->rows);
            if (rows4.x < 0) continue;
            float2 acc_a[kGroupRows], acc_g[kGroupRows];
#pragma unroll
            for (int q = 0; q < kGroupRows; ++q) {
                acc_a[q] = make_float2(bias.x, bias.y);
                acc_g[q] = make_float2(bias.z, bias.w);
            }
            if (overflow)
                accumulate_group<true, BF16W>(grp, feat, wb, lane, hcol, c, acc_a, acc_g);
            else
                accumulate_group<false, BF16W>(grp, feat, wb, lane, hcol, c, acc_a, acc_g);
            const int rows[kGroupRows] = {rows4.x, rows4.y, rows4.z, rows4.w};
#pragma unroll
            for (int q = 0; q < kGroupRows; ++q) {
                if (rows[q] < 0) continue;
                // the conv output is rounded to bf16 before the SwiGLU reads it
                const float a0 = bf2f(f2bf(acc_a[q].x)), a1 = bf2f(f2bf(acc_a[q].y));
                const float g0 = bf2f(f2bf(acc_g[q].x)), g1 = bf2f(f2bf(acc_g[q].y));
                *reinterpret_cast<__nv_bfloat162*>(ocol + (int64_t)rows[q] * half) =
                    __floats2bfloat162_rn(silu(g0) * a0, silu(g1) * a1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(st));
    }
}

int g_sm_count[64] = {0};

}  // namespace

int dwconv_plan_error_word(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_dwplan_error, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    if (clear) {
        int z = 0;
        if (cudaMemcpyToSymbol(g_dwplan_error, &z, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    }
    return v;
}

}  // namespace vdit

using namespace vdit;

extern "C" size_t vdit_dwconv27_plan_bytes(int64_t n) {
    if (n <= 0) return 0;
    return (size_t)((n + kPlanRows - 1) / kPlanRows) * kBlockPlanBytes;
}

extern "C" int vdit_dwconv27_plan(const int32_t* idx, const int64_t* row_order, int64_t n, void* plan,
                                  size_t plan_bytes, vdit_stream_t stream) {
    if (n < 0 || (n > 0 && (!idx || !row_order || !plan))) return VDIT_ERR_ARG;
    if (n > INT32_MAX) return VDIT_ERR_UNSUPPORTED;
    if (n == 0) return VDIT_OK;
    if (!aligned16(plan)) return VDIT_ERR_ALIGN;
    if (plan_bytes < vdit_dwconv27_plan_bytes(n)) return VDIT_ERR_WORKSPACE;
    const int64_t blocks = (n + kPlanRows - 1) / kPlanRows;
    dwconv_plan_kernel<<<(unsigned)blocks, 512, 0, static_cast<cudaStream_t>(stream)>>>(idx, row_order, n, blocks,
                                                                                        plan);
    count_launches(1);
    return check_launch();
}

static int planned_impl(bool bf16w, const void* h, int64_t n, int32_t c, const void* plan, const float* w,
                        const float* b, void* out, vdit_stream_t stream) {
    if (n < 0 || c <= 0 || (n > 0 && (!h || !plan || !w || !b || !out))) return VDIT_ERR_ARG;
    if (c % kTileCols) return VDIT_ERR_UNSUPPORTED;
    if (n == 0) return VDIT_OK;
    if (n > INT32_MAX) return VDIT_ERR_UNSUPPORTED;
    if (!aligned16(h) || !aligned16(plan) || !aligned16(w) || !aligned16(b) || ((uintptr_t)out & 3u))
        return VDIT_ERR_ALIGN;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        record_cuda_error(e);
        return VDIT_ERR_LAUNCH;
    }
    if (dev < 0 || dev >= 64) return VDIT_ERR_UNSUPPORTED;
    if (g_sm_count[dev] == 0) {
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(dwconv_planned_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(dwconv_planned_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return VDIT_ERR_LAUNCH;
        }
        g_sm_count[dev] = sms;
    }
    auto fn = tc::encode_fn();
    if (!fn) return VDIT_ERR_DRIVER;
    // h' as [n rows, c columns] bf16; one-row boxes of 128 columns (tile::gather4)
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)c, (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)c * 2};
    cuuint32_t box[2] = {kTileCols, 1};
    cuuint32_t es[2] = {1, 1};
    if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(h), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return VDIT_ERR_DRIVER;
    const int64_t blocks = (n + kPlanRows - 1) / kPlanRows;
    const int64_t units = blocks * (c / kTileCols);
    const int grid = (int)(units < g_sm_count[dev] ? units : g_sm_count[dev]);
    if (bf16w)
        dwconv_planned_kernel<true><<<grid, (kWarps + 1) * 32, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(
            m, static_cast<const __nv_bfloat16*>(h), c, plan, blocks, w, b, static_cast<__nv_bfloat16*>(out));
    else
        dwconv_planned_kernel<false><<<grid, (kWarps + 1) * 32, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(
            m, static_cast<const __nv_bfloat16*>(h), c, plan, blocks, w, b, static_cast<__nv_bfloat16*>(out));
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_dwconv27_swiglu_planned(const void* h, int64_t n, int32_t c, const void* plan, const float* w,
                                            const float* b, void* out, vdit_stream_t stream) {
    return planned_impl(false, h, n, c, plan, w, b, out, stream);
}

extern "C" int vdit_dwconv27_swiglu_planned_bf16w(const void* h, int64_t n, int32_t c, const void* plan,
                                                  const float* w, const float* b, void* out, vdit_stream_t stream) {
    return planned_impl(true, h, n, c, plan, w, b, out, stream);
}
