// Row-wise fused kernels of the DiT block: AdaLN modulation, gate-add,
// QK-RMSNorm + RoPE (+ Hilbert gather), packed SwiGLU, patchify, output
// modulation + unpatchify, and the small sampler kernels.  All are HBM-bound:
// rows move through registers/shared memory in 16-byte vectors, statistics
// are reduced with warp shuffles in fp32.
#include <algorithm>

#include "common.cuh"
#include "tc.cuh"

namespace vdit {

__device__ int g_rowops_error = 0;

namespace {

constexpr int kRowWarps = 8;            // rows per 256-thread block
constexpr int kMaxVec = 8;              // 16-byte vectors per lane -> d <= 2048

// ---------------------------------------------------------------- LN helpers
// One warp per row; lane l holds vectors l, l+32, ... of the row (8 values each).
struct RowRegs {
    float v[kMaxVec][8];
};

__device__ __forceinline__ void row_load(const __nv_bfloat16* __restrict__ row, int nvec, int lane, RowRegs& r) {
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        int vi = lane + 32 * i;
        if (vi < nvec) load8(row + vi * 8, r.v[i]);
    }
}

// Mean and 1/sqrt(var + 1e-6) of a row, two-pass.  A lane's values are summed in four
// interleaved partial sums (element j of each vector into sum j % 4, combined as (s0 + s1) +
// (s2 + s3)), which keeps four independent add chains in flight instead of one.
__device__ __forceinline__ float sum4(const float (&s)[4]) { return (s[0] + s[1]) + (s[2] + s[3]); }

__device__ __forceinline__ void row_stats(const RowRegs& r, int nvec, int lane, int d, float& mean, float& rstd) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i)
        if (lane + 32 * i < nvec)
#pragma unroll
            for (int j = 0; j < 8; ++j) s[j & 3] += r.v[i][j];
    mean = warp_sum(sum4(s)) / (float)d;
    float q[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i)
        if (lane + 32 * i < nvec)
#pragma unroll
            for (int j = 0; j < 8; ++j) { float t = r.v[i][j] - mean; q[j & 3] += t * t; }
    rstd = rsqrtf(warp_sum(sum4(q)) / (float)d + 1e-6f);
}

__device__ __forceinline__ void row_modulate_store(const RowRegs& r, int nvec, int lane, float mean, float rstd,
                                                   const float* __restrict__ s1, const float* __restrict__ sh,
                                                   __nv_bfloat16* __restrict__ out) {
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        int vi = lane + 32 * i;
        if (vi >= nvec) continue;
        float4 a0 = __ldg(reinterpret_cast<const float4*>(s1 + vi * 8));
        float4 a1 = __ldg(reinterpret_cast<const float4*>(s1 + vi * 8 + 4));
        float4 b0 = __ldg(reinterpret_cast<const float4*>(sh + vi * 8));
        float4 b1 = __ldg(reinterpret_cast<const float4*>(sh + vi * 8 + 4));
        float sa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        float sb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (r.v[i][j] - mean) * rstd * sa[j] + sb[j];
        store8(out + vi * 8, o);
    }
}

__global__ void __launch_bounds__(256) modulate_kernel(const __nv_bfloat16* __restrict__ x, int64_t m, int d,
                                                       const float* __restrict__ s1, const float* __restrict__ sh,
                                                       __nv_bfloat16* __restrict__ out) {
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t row = blockIdx.x * (int64_t)kRowWarps + warp;
    if (row >= m) return;
    int nvec = d >> 3;
    RowRegs r;
    row_load(x + row * d, nvec, lane, r);
    float mean, rstd;
    row_stats(r, nvec, lane, d, mean, rstd);
    row_modulate_store(r, nvec, lane, mean, rstd, s1, sh, out + row * d);
}

// x <- bf16(x + h * g); optional mod_out = LN(x) * s1 + sh
__global__ void __launch_bounds__(256) gate_add_modulate_kernel(
    __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ h, int64_t h_stride, int64_t m, int d,
    const float* __restrict__ g, const __nv_bfloat16* __restrict__ c2, const float* __restrict__ g2,
    const float* __restrict__ s1, const float* __restrict__ sh, __nv_bfloat16* __restrict__ mod_out) {
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t row = blockIdx.x * (int64_t)kRowWarps + warp;
    if (row >= m) return;
    int nvec = d >> 3;
    RowRegs r;
    __nv_bfloat16* xr = x + row * d;
    const __nv_bfloat16* hr = h + row * h_stride;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        int vi = lane + 32 * i;
        if (vi >= nvec) continue;
        float xv[8], hv[8];
        load8(xr + vi * 8, xv);
        load8(hr + vi * 8, hv);
        float4 g0 = __ldg(reinterpret_cast<const float4*>(g + vi * 8));
        float4 g1 = __ldg(reinterpret_cast<const float4*>(g + vi * 8 + 4));
        float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        float cv[8], gv2[8];
        if (c2) {
            load8_nc(c2 + vi * 8, cv);
            const float4 a0 = __ldg(reinterpret_cast<const float4*>(g2 + vi * 8));
            const float4 a1 = __ldg(reinterpret_cast<const float4*>(g2 + vi * 8 + 4));
            const float t8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) gv2[j] = t8[j];
        }
        uint4 packed;
        __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            p2[j] = __floats2bfloat162_rn(xv[2 * j] + hv[2 * j] * gg[2 * j], xv[2 * j + 1] + hv[2 * j + 1] * gg[2 * j + 1]);
            float2 t = __bfloat1622float2(p2[j]);
            if (c2) {       // second residual, rounded like a second gate-add pass
                p2[j] = __floats2bfloat162_rn(t.x + cv[2 * j] * gv2[2 * j], t.y + cv[2 * j + 1] * gv2[2 * j + 1]);
                t = __bfloat1622float2(p2[j]);
            }
            r.v[i][2 * j] = t.x;
            r.v[i][2 * j + 1] = t.y;
        }
        *reinterpret_cast<uint4*>(xr + vi * 8) = packed;
    }
    if (mod_out == nullptr) return;
    float mean, rstd;
    row_stats(r, nvec, lane, d, mean, rstd);
    row_modulate_store(r, nvec, lane, mean, rstd, s1, sh, mod_out + row * d);
}

// The same operation as gate_add_modulate_kernel from persistent CTAs: one CTA
// per SM stages g, s1, sh in shared memory once, and each warp walks rows with
// a stride, bulk-copying the next row's x and h into its second buffer while
// the current row is reduced and written.  With h == nullptr the kernel is the
// plain modulation (modulate_kernel): only x is copied, into a four-row ring
// (three rows in flight per warp, the same bytes in flight as with the
// residual), and x is not written.
// Arithmetic is identical to the one-row-per-warp kernels.  Waits on the bulk
// copies are bounded; a timeout sets the row kernels' error word.
constexpr int kGaMaxWarps = 16;
constexpr int kGaVecBytes = 20;          // shared fp32 vectors per column: g, s1, sh, g2, c2
constexpr int kGaSlots = 4;              // row slots per warp (an even number)
constexpr int kErrRowTimeout = 0x524f;   // "RO": a bounded wait of a row kernel ran out

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__global__ void __launch_bounds__(kGaMaxWarps * 32, 1) gate_add_modulate_staged_kernel(
    __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ h, int64_t h_stride, int64_t m, int d,
    const float* __restrict__ g, const __nv_bfloat16* __restrict__ c2, const float* __restrict__ g2,
    const float* __restrict__ s1, const float* __restrict__ sh, __nv_bfloat16* __restrict__ mod_out) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    const int nwarps = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool mod = mod_out != nullptr;
    const bool add = h != nullptr;
    float* pg = reinterpret_cast<float*>(smem);
    float* ps1 = pg + d;
    float* psh = ps1 + d;
    float* pg2 = psh + d;            // second residual: its gate and its (broadcast) row in fp32
    float* pc2 = pg2 + d;
    const uint32_t row_bytes = 2u * (uint32_t)d;
    // a warp's row slots: stages of [x | h] with the residual, else stages of x alone
    const int nst = add ? kGaSlots / 2 : kGaSlots;
    uint8_t* wbuf = smem + (size_t)kGaVecBytes * d + (size_t)warp * kGaSlots * row_bytes;
    uint64_t* bars =
        reinterpret_cast<uint64_t*>(smem + (size_t)kGaVecBytes * d + (size_t)nwarps * kGaSlots * row_bytes) +
        warp * kGaSlots;
    const uint32_t bar0 = tc::smem_u32(bars);
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        if (add) pg[i] = g[i];
        if (mod) {
            ps1[i] = s1[i];
            psh[i] = sh[i];
        }
        if (c2) {
            pg2[i] = g2[i];
            pc2[i] = bf2f(c2[i]);
        }
    }
    if (threadIdx.x == 0) abort_flag = 0;
    if (lane == 0) {
        for (int b = 0; b < nst; ++b) tc::mbar_init(bar0 + 8 * b, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const int nvec = d >> 3;
    const int64_t stride = (int64_t)gridDim.x * nwarps;
    const int slot_rows = add ? 2 : 1;
    auto issue = [&](int64_t row, int b) {
        const uint32_t dst = tc::smem_u32(wbuf + b * slot_rows * row_bytes);
        tc::mbar_expect_tx(bar0 + 8 * b, slot_rows * row_bytes);
        bulk_load(dst, x + row * d, row_bytes, bar0 + 8 * b);
        if (add) bulk_load(dst + row_bytes, h + row * h_stride, row_bytes, bar0 + 8 * b);
    };
    int64_t row = (int64_t)blockIdx.x * nwarps + warp;
    if (lane == 0)
        for (int k = 0; k < nst - 1; ++k)
            if (row + k * stride < m) issue(row + k * stride, k);
    int it = 0;
    bool ok = true;
    for (; row < m; row += stride, ++it) {
        const int b = it % nst;
        // the row nst - 1 ahead goes into the buffer read in the previous iteration
        if (lane == 0 && row + (nst - 1) * stride < m) issue(row + (nst - 1) * stride, (it + nst - 1) % nst);
        ok = __all_sync(0xffffffffu, tc::mbar_wait(bar0 + 8 * b, (it / nst) & 1, &abort_flag, &g_rowops_error,
                                                   kErrRowTimeout));
        if (!ok) break;
        const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(wbuf + b * slot_rows * row_bytes);
        const __nv_bfloat16* hs = xs + d;
        __nv_bfloat16* xr = x + row * d;
        RowRegs r;
        if (!add) {
            row_load(xs, nvec, lane, r);
        }
#pragma unroll
        for (int i = 0; i < kMaxVec; ++i) {
            const int vi = lane + 32 * i;
            if (!add || vi >= nvec) continue;
            float xv[8], hv[8];
            load8(xs + vi * 8, xv);
            load8(hs + vi * 8, hv);
            const float4 g0 = *reinterpret_cast<const float4*>(pg + vi * 8);
            const float4 g1 = *reinterpret_cast<const float4*>(pg + vi * 8 + 4);
            const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            float cc[8], gc[8];              // second residual's row and gate (16-byte reads)
            if (c2) {
                const float4 c0 = *reinterpret_cast<const float4*>(pc2 + vi * 8);
                const float4 c1 = *reinterpret_cast<const float4*>(pc2 + vi * 8 + 4);
                const float4 q0 = *reinterpret_cast<const float4*>(pg2 + vi * 8);
                const float4 q1 = *reinterpret_cast<const float4*>(pg2 + vi * 8 + 4);
                cc[0] = c0.x; cc[1] = c0.y; cc[2] = c0.z; cc[3] = c0.w;
                cc[4] = c1.x; cc[5] = c1.y; cc[6] = c1.z; cc[7] = c1.w;
                gc[0] = q0.x; gc[1] = q0.y; gc[2] = q0.z; gc[3] = q0.w;
                gc[4] = q1.x; gc[5] = q1.y; gc[6] = q1.z; gc[7] = q1.w;
            }
            uint4 packed;
            __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                p2[j] = __floats2bfloat162_rn(xv[2 * j] + hv[2 * j] * gg[2 * j],
                                              xv[2 * j + 1] + hv[2 * j + 1] * gg[2 * j + 1]);
                float2 t = __bfloat1622float2(p2[j]);
                if (c2) {   // second residual, rounded like a second gate-add pass
                    p2[j] = __floats2bfloat162_rn(t.x + cc[2 * j] * gc[2 * j], t.y + cc[2 * j + 1] * gc[2 * j + 1]);
                    t = __bfloat1622float2(p2[j]);
                }
                r.v[i][2 * j] = t.x;
                r.v[i][2 * j + 1] = t.y;
            }
            *reinterpret_cast<uint4*>(xr + vi * 8) = packed;
        }
        __syncwarp();                                    // this buffer may be refilled after the next wait
        if (!mod) continue;
        float mean, rstd;
        row_stats(r, nvec, lane, d, mean, rstd);
        __nv_bfloat16* orow = mod_out + row * d;
#pragma unroll
        for (int i = 0; i < kMaxVec; ++i) {
            const int vi = lane + 32 * i;
            if (vi >= nvec) continue;
            const float4 a0 = *reinterpret_cast<const float4*>(ps1 + vi * 8);
            const float4 a1 = *reinterpret_cast<const float4*>(ps1 + vi * 8 + 4);
            const float4 b0 = *reinterpret_cast<const float4*>(psh + vi * 8);
            const float4 b1 = *reinterpret_cast<const float4*>(psh + vi * 8 + 4);
            const float sa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float sb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            float o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = (r.v[i][j] - mean) * rstd * sa[j] + sb[j];
            store8(orow + vi * 8, o);
        }
    }
    if (lane == 0 && !ok) {
        // a wait ran out: give the copies still in flight (rows it .. it + nst - 1) time to land
        volatile int no_abort = 0;
        for (int k = it; k < it + nst; ++k)
            if (row + (k - it) * stride < m)
                tc::mbar_wait(bar0 + 8 * (k % nst), (k / nst) & 1, &no_abort, &g_rowops_error, kErrRowTimeout);
    }
}

// out[row, o] = sum_c y[row, c] * w[o, c] with y = bf16(LN(x[row]) * s1 + sh) and fp32 weights
// w [16, d]: 16 fp32 outputs per row, on the tensor cores at fp32 accuracy.  Each weight is split
// into three bf16 parts, hi = bf16(w), mid = bf16(w - hi), lo = bf16(w - hi - mid): both
// differences are exact in fp32 and hi + mid + lo carries w's 24-bit significand.  B = [hi; mid;
// lo] is then a 48 x d bf16 matrix, every product y * part (bf16 x bf16) is exact in the fp32
// accumulator, and one M=128, N=48 MMA chain gives the three partial sums of each output, which
// the epilogue adds (lo + mid first).
// A CTA takes 128 rows.  Phase 1: warps 0-7 compute the rows' LayerNorm statistics with the sums
// of row_stats (16 rows per warp), the one HBM read of x: each warp streams its rows through a
// ring of up to six row slots filled by bulk copies (the stage buffers, idle until phase 2), so
// five rows stay in flight while one is reduced.  Phase 2: per 64-column chunk the warps read the
// chunk again (from L2), modulate it into a 128-row x 128-byte stage in the 128-byte-swizzled
// K-major layout of the MMA's A operand (16-byte piece c of row r at (r / 8) * 1024 + (r % 8) *
// 128 + ((c ^ r % 8) * 16)), and write the chunk's split weights into the stage's B part in the
// same layout; four chunks are prepared per round, their row and weight loads issued together,
// each chunk on its own stage of an eight-stage ring, with s1 and sh read from shared memory.
// Warp 8 issues each chunk's four K=16 MMAs and frees the stage with a commit.  Warps 0-3 read the
// 128 x 48 accumulator back from TMEM and store the 16 outputs of a row.
constexpr int kUpRows = 128;                                   // rows per CTA (the MMA's M)
constexpr int kUpK = 64;                                       // columns per chunk (128 bytes of bf16)
constexpr int kUpN = 48;                                       // hi, mid and lo parts of 16 outputs
constexpr int kUpStages = 8;
constexpr int kUpRound = 4;                                    // chunks prepared per round
constexpr int kUpWarps = 8;                                    // + warp 8, the MMA issuer
constexpr int kUpSlots = 6;                                    // phase-1 row slots per warp (at most)
constexpr int kUpMaxD = 256 * kMaxVec;
constexpr int kUpABytes = kUpRows * 128;
constexpr int kUpStageBytes = kUpABytes + kUpN * 128;          // 22 KB, a multiple of 1024
constexpr int kUpBarOff = kUpStages * kUpStageBytes;           // phase-2 barriers, TMEM slot, abort flag
constexpr int kUpRowBarOff = kUpBarOff + 256;                  // phase-1 slot barriers
constexpr int kUpStatsOff = kUpRowBarOff + kUpWarps * kUpSlots * 8;
constexpr int kUpVecOff = kUpStatsOff + kUpRows * 8;           // s1, sh as fp32
constexpr int kUpSmem = 1024 + kUpVecOff + 2 * kUpMaxD * 4;    // 1024: alignment slack
constexpr int kErrUnpTimeout = 0x5550;                         // "UP": a bounded wait ran out
static_assert(kUpStageBytes % 1024 == 0 && kUpStages % kUpRound == 0, "stage layout");
static_assert((2 * kUpStages + 1) * 8 + 8 <= 256, "barrier area");
static_assert(kUpSmem <= 227 * 1024, "shared memory per CTA");

__device__ __forceinline__ uint32_t up_swz(int r, int c) {      // byte offset of 16-byte piece c of row r
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// VEC: 16-byte vectors per lane of a row in phase 1 (d <= 256 VEC)
template <int VEC>
__global__ void __launch_bounds__((kUpWarps + 1) * 32, 1) out_unpatchify_kernel(
        const __nv_bfloat16* __restrict__ x, int64_t m, int d, const float* __restrict__ s1,
        const float* __restrict__ sh, const float* __restrict__ w, float* __restrict__ out) {
    using namespace tc;
    extern __shared__ uint8_t up_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(up_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kUpBarOff);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kUpStages + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float2* stats = reinterpret_cast<float2*>(sm + kUpStatsOff);
    float* s1_s = reinterpret_cast<float*>(sm + kUpVecOff);
    float* sh_s = s1_s + kUpMaxD;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t row0 = (int64_t)blockIdx.x * kUpRows;
    const int nvec = d >> 3;
    const int nk = (d + kUpK - 1) / kUpK;
    const uint32_t row_bytes = 2u * (uint32_t)d;
    const int nslot = min(kUpSlots, kUpBarOff / (kUpWarps * (int)row_bytes));
    auto full = [&](int s) { return smem_u32(&bars[s]); };
    auto empty = [&](int s) { return smem_u32(&bars[kUpStages + s]); };
    const uint32_t done = smem_u32(&bars[2 * kUpStages]);
    const uint32_t rbar0 = smem_u32(sm + kUpRowBarOff) + warp * kUpSlots * 8;

    if (tid == 0) {
        for (int s = 0; s < kUpStages; ++s) {
            mbar_init(full(s), kUpWarps);
            mbar_init(empty(s), 1);
        }
        mbar_init(done, 1);
        for (int k = 0; k < kUpWarps * kUpSlots; ++k) mbar_init(smem_u32(sm + kUpRowBarOff) + 8 * k, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = tid; i < d; i += blockDim.x) {
        s1_s[i] = s1[i];
        sh_s[i] = sh[i];
    }
    __syncthreads();
    if (warp == kUpWarps) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 64;" ::"r"(smem_u32(tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    } else {
        // ---------------- phase 1: LayerNorm statistics of rows 16 warp .. 16 warp + 15
        const int rw = warp * 16;
        const int64_t left = m - row0 - rw;
        const int nr = left <= 0 ? 0 : (left >= 16 ? 16 : (int)left);   // live rows of this warp
        uint8_t* ring = sm + (size_t)warp * nslot * row_bytes;
        auto issue = [&](int i) {
            const uint32_t bar = rbar0 + 8 * (i % nslot);
            mbar_expect_tx(bar, row_bytes);
            bulk_load(smem_u32(ring + (i % nslot) * row_bytes), x + (row0 + rw + i) * d, row_bytes, bar);
        };
        if (lane == 0)
            for (int i = 0; i < nslot && i < nr; ++i) issue(i);
        int i = 0;
        bool ok = true;
        for (; i < nr; ++i) {
            ok = __all_sync(0xffffffffu, mbar_wait(rbar0 + 8 * (i % nslot), (i / nslot) & 1, abort_flag,
                                                   &g_rowops_error, kErrUnpTimeout));
            if (!ok) break;
            const uint4* xs = reinterpret_cast<const uint4*>(ring + (i % nslot) * row_bytes);
            uint4 y[VEC];
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
                const int vi = lane + 32 * v;
                y[v] = vi < nvec ? xs[vi] : make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();                                  // the slot may be refilled now
            if (lane == 0 && i + nslot < nr) issue(i + nslot);
            float sum[4] = {0.f, 0.f, 0.f, 0.f};       // the partial sums of row_stats
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
                if (lane + 32 * v >= nvec) continue;
                float f[8];
                unpack8(y[v], f);
#pragma unroll
                for (int j = 0; j < 8; ++j) sum[j & 3] += f[j];
            }
            const float mean = warp_sum(sum4(sum)) / (float)d;
            float sq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
                if (lane + 32 * v >= nvec) continue;
                float f[8];
                unpack8(y[v], f);
#pragma unroll
                for (int j = 0; j < 8; ++j) { const float t = f[j] - mean; sq[j & 3] += t * t; }
            }
            const float rstd = rsqrtf(warp_sum(sum4(sq)) / (float)d + 1e-6f);
            if (lane == 0) stats[rw + i] = make_float2(mean, rstd);
        }
        if (lane == 0 && !ok) {
            // a wait ran out: let the copies still in flight land before the slots are reused
            volatile int no_abort = 0;
            for (int k = i; k < nr && k < i + nslot; ++k)
                mbar_wait(rbar0 + 8 * (k % nslot), (k / nslot) & 1, &no_abort, &g_rowops_error, kErrUnpTimeout);
        }
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < kUpWarps) {
        // ---------------- phase 2 producers: thread tid owns 16-byte piece c = tid % 8 of rows
        // tid / 8 + 32 h (h = 0..3) of every chunk, and splits 4 of the chunk's 16 x 64 weights
        const int c = tid & 7, rr = tid >> 3;
        const int wo = tid >> 4, wq = tid & 15;
        float2 st[4];
        const __nv_bfloat16* xr[4];
        bool live[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            live[h] = row0 + rr + 32 * h < m;
            st[h] = stats[rr + 32 * h];
            xr[h] = x + (live[h] ? row0 + rr + 32 * h : 0) * d;
        }
        bool ok = !*abort_flag;
#pragma unroll 1
        for (int k0 = 0; ok && k0 < nk; k0 += kUpRound) {
            uint4 raw[kUpRound][4];
            float4 wv[kUpRound];
#pragma unroll
            for (int g = 0; g < kUpRound; ++g) {
                const int col = (k0 + g) * kUpK + 8 * c;
                const bool cok = k0 + g < nk && col < d;
#pragma unroll
                for (int h = 0; h < 4; ++h)
                    raw[g][h] = (cok && live[h]) ? __ldg(reinterpret_cast<const uint4*>(xr[h] + col))
                                                 : make_uint4(0u, 0u, 0u, 0u);
                const int wc = (k0 + g) * kUpK + 4 * wq;
                wv[g] = (k0 + g < nk && wc < d) ? __ldg(reinterpret_cast<const float4*>(w + (int64_t)wo * d + wc))
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int g = 0; g < kUpRound; ++g) {
                const int k = k0 + g;
                if (k >= nk) break;
                const int s = k % kUpStages;
                if (k >= kUpStages &&
                    !__all_sync(0xffffffffu, mbar_wait(empty(s), ((k / kUpStages) - 1) & 1, abort_flag,
                                                       &g_rowops_error, kErrUnpTimeout))) {
                    ok = false;
                    break;
                }
                uint8_t* stg = sm + s * kUpStageBytes;
                const int col = k * kUpK + 8 * c;
                if (col < d) {
                    const float4 a0 = *reinterpret_cast<const float4*>(s1_s + col);
                    const float4 a1 = *reinterpret_cast<const float4*>(s1_s + col + 4);
                    const float4 b0 = *reinterpret_cast<const float4*>(sh_s + col);
                    const float4 b1 = *reinterpret_cast<const float4*>(sh_s + col + 4);
                    const float sa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    const float sb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        uint4 v = make_uint4(0u, 0u, 0u, 0u);
                        if (live[h]) {
                            float f[8];
                            unpack8(raw[g][h], f);
#pragma unroll
                            for (int j = 0; j < 8; ++j) f[j] = (f[j] - st[h].x) * st[h].y * sa[j] + sb[j];
                            v = pack8(f);
                        }
                        *reinterpret_cast<uint4*>(stg + up_swz(rr + 32 * h, c)) = v;
                    }
                } else {
#pragma unroll
                    for (int h = 0; h < 4; ++h)
                        *reinterpret_cast<uint4*>(stg + up_swz(rr + 32 * h, c)) = make_uint4(0u, 0u, 0u, 0u);
                }
                {
                    // weights w[wo, 4 wq .. 4 wq + 3] of the chunk -> B rows wo, 16 + wo, 32 + wo
                    float r[4] = {wv[g].x, wv[g].y, wv[g].z, wv[g].w};
#pragma unroll
                    for (int part = 0; part < 3; ++part) {
                        __nv_bfloat162 lo2 = __floats2bfloat162_rn(r[0], r[1]), hi2 = __floats2bfloat162_rn(r[2], r[3]);
                        r[0] -= __low2float(lo2);
                        r[1] -= __high2float(lo2);
                        r[2] -= __low2float(hi2);
                        r[3] -= __high2float(hi2);
                        const int n = 16 * part + wo;
                        uint2 pk;
                        pk.x = *reinterpret_cast<uint32_t*>(&lo2);
                        pk.y = *reinterpret_cast<uint32_t*>(&hi2);
                        *reinterpret_cast<uint2*>(stg + kUpABytes + up_swz(n, wq >> 1) + (wq & 1) * 8) = pk;
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor core
                __syncwarp();
                if (lane == 0) mbar_arrive(full(s));
            }
        }
    } else {
        // ---------------- MMA issuer (converged warp, elected lane)
        const uint64_t a0 = make_desc(smem_u32(sm), 16, 1024, kSw128);
        const uint64_t b0 = make_desc(smem_u32(sm + kUpABytes), 16, 1024, kSw128);
        constexpr uint32_t kIdesc = make_idesc(kUpRows, kUpN, false);
        bool ok = true;
        for (int k = 0; k < nk; ++k) {
            const int s = k % kUpStages;
            if (!__all_sync(0xffffffffu, mbar_wait(full(s), (k / kUpStages) & 1, abort_flag, &g_rowops_error,
                                                   kErrUnpTimeout))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint64_t so = (uint64_t)(s * (kUpStageBytes >> 4));
#pragma unroll
            for (int kk = 0; kk < kUpK / 16; ++kk)
                tc_mma_elect(tmem, a0 + so + kk * 2, b0 + so + kk * 2, kIdesc, (k > 0 || kk > 0) ? 1u : 0u);
            tc_commit_elect(empty(s));
        }
        if (ok) tc_commit_elect(done);
    }

    // ---------------- epilogue: warp q reads TMEM lanes 32q .. 32q + 31 (the tile's rows)
    if (warp < 4) {
        if (__all_sync(0xffffffffu, mbar_wait(done, 0, abort_flag, &g_rowops_error, kErrUnpTimeout))) {
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
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kUpWarps) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 64;" ::"r"(tmem));
    }
}

// ---------------------------------------------------------------- QK norm + RoPE
// One warp per token row, looping over its heads: lanes 0..15 hold a head's q
// vector, lanes 16..31 its k vector (8 channels each, one 16-byte load per lane;
// head_dim 96 uses 12 lanes per half).  The token's source index, coordinates
// and the RoPE cos/sin of each lane's 8 channels are fetched once and reused
// for every head; the next head's vectors are loaded while the current one is
// normalised.  RMS statistics reduce over the 16-lane half with shuffles; the
// normalised values go through a per-warp shared-memory slot so each lane can
// read its RoPE partner channel (e +- M); v is copied through.
//   MODE 0: 3D RoPE, positions from h_coords[src] via the [res, hd/6] tables,
//           optional gather src = fwd[dst].
//   MODE 1: 2D RoPE on tokens >= n_prefix via [L-n_prefix, 2, hd/4] tables, in place.
constexpr int kQkWarps = 8;

template <int MODE>
__global__ void __launch_bounds__(kQkWarps * 32) qknorm_rope_kernel(
    const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int64_t rows, int heads, int hd,
    const float* __restrict__ qs, const float* __restrict__ ks, const float* __restrict__ cs,
    const float* __restrict__ sn, int res, const int4* __restrict__ hc, const int64_t* __restrict__ fwd,
    int n_prefix) {
    __shared__ float snorm[kQkWarps][2][128];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t dst = (int64_t)blockIdx.x * kQkWarps + warp;
    if (dst >= rows) return;
    const int64_t src = (MODE == 0 && fwd != nullptr) ? fwd[dst] : dst;
    const int D = heads * hd;
    const int half = lane >> 4, vi = lane & 15;                 // half 0 = q, 1 = k
    const bool active = vi * 8 < hd;
    const __nv_bfloat16* irow = in + src * (int64_t)(3 * D);
    __nv_bfloat16* orow = out + dst * (int64_t)(3 * D);

    // RoPE of this lane's 8 channels (identical for every head)
    const int naxes = MODE == 0 ? 3 : 2;
    const int M = hd / (2 * naxes);
    bool rotate = true;
    int64_t tab_row[3] = {0, 0, 0};
    if (MODE == 0) {
        const int4 c = hc[src];
        tab_row[0] = min(max(c.y, 0), res - 1);
        tab_row[1] = min(max(c.z, 0), res - 1);
        tab_row[2] = min(max(c.w, 0), res - 1);
    } else {
        rotate = dst >= n_prefix;
        const int64_t pt = dst - n_prefix;
        tab_row[0] = pt * 2;
        tab_row[1] = pt * 2 + 1;
    }
    float rc[8], rs[8];
    int partner[8];            // channel index of the RoPE partner, -1: channel passes through
    bool lower[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int e = vi * 8 + j;
        const int grp = e / (2 * M), off = e - grp * 2 * M;
        rc[j] = 1.f;
        rs[j] = 0.f;
        partner[j] = -1;
        lower[j] = true;
        if (active && rotate && grp < naxes) {
            const int f = off < M ? off : off - M;
            rc[j] = __ldg(cs + tab_row[grp] * M + f);
            rs[j] = __ldg(sn + tab_row[grp] * M + f);
            lower[j] = off < M;
            partner[j] = lower[j] ? e + M : e - M;
        }
    }

    float* nb = snorm[warp][half];
    float x[8] = {0, 0, 0, 0, 0, 0, 0, 0};        // lanes past head_dim must add zeros to the RMS sum
    uint4 vcopy = make_uint4(0, 0, 0, 0);
    if (active) {
        load8(irow + half * D + vi * 8, x);
        if (half == 0) vcopy = *reinterpret_cast<const uint4*>(irow + 2 * D + vi * 8);
    }
    for (int h = 0; h < heads; ++h) {
        // prefetch the next head's vectors
        float xn[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        uint4 vn = make_uint4(0, 0, 0, 0);
        if (active && h + 1 < heads) {
            load8(irow + half * D + (h + 1) * hd + vi * 8, xn);
            if (half == 0) vn = *reinterpret_cast<const uint4*>(irow + 2 * D + (h + 1) * hd + vi * 8);
        }
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rr = rsqrtf(ss / (float)hd + 1e-6f);
        const float* scale = (half == 0 ? qs : ks) + h * hd;
        __syncwarp();                                    // the previous head's partner reads are done
        if (active) {
            const float4 s0 = __ldg(reinterpret_cast<const float4*>(scale + vi * 8));
            const float4 s1 = __ldg(reinterpret_cast<const float4*>(scale + vi * 8 + 4));
            const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                x[j] = bf2f(f2bf(x[j] * rr)) * sc[j];        // normalised value rounded like the reference
                nb[vi * 8 + j] = x[j];
            }
        }
        __syncwarp();
        if (active) {
            float o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                o[j] = x[j];
                if (partner[j] >= 0) {
                    const float pv = nb[partner[j]];
                    o[j] = lower[j] ? x[j] * rc[j] - pv * rs[j] : x[j] * rc[j] + pv * rs[j];
                }
            }
            store8(orow + half * D + h * hd + vi * 8, o);
            if (half == 0) *reinterpret_cast<uint4*>(orow + 2 * D + h * hd + vi * 8) = vcopy;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = xn[j];
        vcopy = vn;
    }
}

// ---------------------------------------------------------------- context vector (1-token branch)
// out = bf16(LN(v) * s1 + sh) for one fp32 vector (d <= 2048): one block, two-pass
// statistics (mean, then mean of squared deviations) in fp32.
__global__ void __launch_bounds__(256) vec_ln_modulate_kernel(const float* __restrict__ v, int d,
                                                              const float* __restrict__ s1,
                                                              const float* __restrict__ sh,
                                                              __nv_bfloat16* __restrict__ out) {
    __shared__ float red[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float x[8];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int i = tid + 256 * k;
        x[k] = i < d ? v[i] : 0.f;
        s += x[k];
    }
    auto block_sum = [&](float t) {
        t = warp_sum(t);
        __syncthreads();
        if (lane == 0) red[warp] = t;
        __syncthreads();
        float r = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) r += red[w];
        return r;
    };
    const float mean = block_sum(s) / (float)d;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
        if (tid + 256 * k < d) q += (x[k] - mean) * (x[k] - mean);
    const float rstd = rsqrtf(block_sum(q) / (float)d + 1e-6f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int i = tid + 256 * k;
        if (i < d) out[i] = f2bf((x[k] - mean) * rstd * s1[i] + sh[i]);
    }
}

// c += float(y) * g for one fp32 vector and a bf16 update
__global__ void vec_gate_residual_kernel(float* __restrict__ c, const __nv_bfloat16* __restrict__ y,
                                         const float* __restrict__ g, int d) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < d) c[i] += bf2f(y[i]) * g[i];
}

// ---------------------------------------------------------------- misc
__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ h, int64_t m, int f, __nv_bfloat16* __restrict__ out) {
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int fv = f >> 3;
    if (t >= m * fv) return;
    int64_t row = t / fv;
    int c = (int)(t % fv) * 8;
    float a[8], g[8], o[8];
    load8(h + row * 2 * f + c, a);
    load8(h + row * 2 * f + f + c, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = silu(g[j]) * a[j];
    store8(out + row * f + c, o);
}

__global__ void gather_rows_f32_kernel(const float* __restrict__ src, const int64_t* __restrict__ idx, int64_t n, int c,
                                       float* __restrict__ dst) {
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (t >= n * c) return;
    int64_t r = t / c;
    dst[t] = src[idx[r] * c + (t % c)];
}

__global__ void cfg_euler_kernel(float* __restrict__ xt, const float* __restrict__ vp, const float* __restrict__ vn,
                                 int64_t total, float g, float dt) {
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (t >= total) return;
    float v = vp[t];
    if (vn) v = v + g * (v - vn[t]);
    xt[t] = xt[t] - dt * v;
}

__global__ void unpermute_denorm_kernel(const float* __restrict__ xt, const int64_t* __restrict__ up, int64_t n,
                                        const float* __restrict__ sc, const float* __restrict__ shf, float* __restrict__ out) {
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (t >= n * 16) return;
    int64_t i = t >> 4;
    int c = (int)(t & 15);
    out[t] = xt[up[i] * 16 + c] * sc[c] + shf[c];
}

inline unsigned blocks_for(int64_t n, int per) { return (unsigned)((n + per - 1) / per); }

}  // namespace

int rowops_error_word(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_rowops_error, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    if (clear) {
        int z = 0;
        if (cudaMemcpyToSymbol(g_rowops_error, &z, sizeof(int)) != cudaSuccess) return VDIT_ERR_LAUNCH;
    }
    return v;
}

}  // namespace vdit

using namespace vdit;

static bool row_width_ok(int32_t d) { return d > 0 && d % 8 == 0 && d <= 256 * kMaxVec; }

int launch_gate_add_staged(__nv_bfloat16* x, const __nv_bfloat16* h, int64_t h_stride, int64_t m, int d,
                           const float* g, const __nv_bfloat16* c2, const float* g2, const float* s1, const float* sh,
                           __nv_bfloat16* mod_out, cudaStream_t s) {
    static int sms[64] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        if (e != cudaSuccess) record_cuda_error(e);
        return VDIT_ERR_LAUNCH;
    }
    constexpr size_t kMaxSmem = 227 * 1024 - 256;
    const size_t per_warp = (size_t)kGaSlots * (2 * d + 8);   // row slots and their barriers
    const int nwarps = (int)std::min<size_t>(kGaMaxWarps, (kMaxSmem - (size_t)kGaVecBytes * d) / per_warp);
    if (sms[dev] == 0) {
        int n = 0;
        e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gate_add_modulate_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kMaxSmem);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return VDIT_ERR_LAUNCH;
        }
        sms[dev] = n;
    }
    const size_t smem = (size_t)kGaVecBytes * d + (size_t)nwarps * per_warp;
    const unsigned grid = (unsigned)std::min<int64_t>((m + nwarps - 1) / nwarps, sms[dev]);
    gate_add_modulate_staged_kernel<<<grid, nwarps * 32, smem, s>>>(x, h, h_stride, m, d, g, c2, g2, s1, sh, mod_out);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_modulate(const void* x, int64_t m, int32_t d, const float* s1, const float* sh, void* out,
                             vdit_stream_t stream) {
    if (m < 0 || !row_width_ok(d) || !x || !s1 || !sh || !out) return VDIT_ERR_ARG;
    if (!aligned16(x) || !aligned16(out) || !aligned16(s1) || !aligned16(sh)) return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    if (m >= 4096)       // persistent CTAs with bulk-copied rows (the staged kernel without its gate-add)
        return launch_gate_add_staged(const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(x)), nullptr, 0, m,
                                      d, nullptr, nullptr, nullptr, s1, sh, static_cast<__nv_bfloat16*>(out),
                                      static_cast<cudaStream_t>(stream));
    modulate_kernel<<<blocks_for(m, kRowWarps), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(x), m, d, s1, sh, static_cast<__nv_bfloat16*>(out));
    count_launches(1);
    return check_launch();
}

static int gate_add_impl(void* x, const void* h, int64_t h_stride, int64_t m, int32_t d, const float* g,
                         const void* c2, const float* g2, const float* s1, const float* sh, void* mod_out,
                         vdit_stream_t stream) {
    if (m < 0 || !row_width_ok(d) || !x || !h || !g || h_stride < 0) return VDIT_ERR_ARG;
    if (mod_out && (!s1 || !sh)) return VDIT_ERR_ARG;
    if ((c2 == nullptr) != (g2 == nullptr)) return VDIT_ERR_ARG;
    if (!aligned16(x) || !aligned16(h) || !aligned16(g) || (h_stride % 8) || (mod_out && !aligned16(mod_out)) ||
        (s1 && !aligned16(s1)) || (sh && !aligned16(sh)) || (c2 && !aligned16(c2)) || (g2 && !aligned16(g2)))
        return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    auto* xb = static_cast<__nv_bfloat16*>(x);
    auto* hb = static_cast<const __nv_bfloat16*>(h);
    auto* cb = static_cast<const __nv_bfloat16*>(c2);
    auto* ob = static_cast<__nv_bfloat16*>(mod_out);
    if (m >= 4096)       // enough rows for persistent CTAs to pay off
        return launch_gate_add_staged(xb, hb, h_stride, m, d, g, cb, g2, s1, sh, ob, static_cast<cudaStream_t>(stream));
    gate_add_modulate_kernel<<<blocks_for(m, kRowWarps), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        xb, hb, h_stride, m, d, g, cb, g2, s1, sh, ob);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_gate_add_modulate(void* x, const void* h, int64_t h_stride, int64_t m, int32_t d, const float* g,
                                      const float* s1, const float* sh, void* mod_out, vdit_stream_t stream) {
    return gate_add_impl(x, h, h_stride, m, d, g, nullptr, nullptr, s1, sh, mod_out, stream);
}

extern "C" int vdit_gate_add2_modulate(void* x, const void* h, int64_t h_stride, int64_t m, int32_t d, const float* g,
                                       const void* c2, const float* g2, const float* s1, const float* sh,
                                       void* mod_out, vdit_stream_t stream) {
    if (!c2 || !g2) return VDIT_ERR_ARG;
    return gate_add_impl(x, h, h_stride, m, d, g, c2, g2, s1, sh, mod_out, stream);
}

extern "C" int vdit_out_modulate_unpatchify(const void* x, int64_t m, int32_t d, const float* s1, const float* sh,
                                            const float* w, float* out, vdit_stream_t stream) {
    if (m < 0 || !row_width_ok(d) || !x || !s1 || !sh || !w || !out) return VDIT_ERR_ARG;
    if (!aligned16(x) || !aligned16(w) || !aligned16(s1) || !aligned16(sh) || !aligned16(out)) return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        if (e != cudaSuccess) record_cuda_error(e);
        return VDIT_ERR_LAUNCH;
    }
    if (!attr_set[dev]) {
        e = cudaFuncSetAttribute(out_unpatchify_kernel<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, kUpSmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(out_unpatchify_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kUpSmem);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return VDIT_ERR_LAUNCH;
        }
        attr_set[dev] = true;
    }
    const int64_t tiles = (m + kUpRows - 1) / kUpRows;
    const auto kernel = d <= 256 * 6 ? out_unpatchify_kernel<6> : out_unpatchify_kernel<8>;
    kernel<<<(unsigned)tiles, (kUpWarps + 1) * 32, kUpSmem, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(x), m, d, s1, sh, w, out);
    count_launches(1);
    return check_launch();
}


extern "C" int vdit_qknorm_rope3d_gather(const void* qkv, int64_t n, int32_t heads, int32_t hd, const float* qs,
                                         const float* ks, const float* cs, const float* sn, int32_t res,
                                         const int32_t* h_coords, const int64_t* fwd, void* out, vdit_stream_t stream) {
    if (n < 0 || heads < 1 || hd < 6 || hd % 8 || !qkv || !qs || !ks || !cs || !sn || !h_coords || !out || res < 1)
        return VDIT_ERR_ARG;
    if (qkv == out && fwd != nullptr) return VDIT_ERR_ARG;     // a gather cannot run in place
    if (!aligned16(qkv) || !aligned16(out) || !aligned16(h_coords)) return VDIT_ERR_ALIGN;
    if (n == 0) return VDIT_OK;
    if (hd > 128) return VDIT_ERR_UNSUPPORTED;
    qknorm_rope_kernel<0><<<blocks_for(n, kQkWarps), kQkWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(out), n, heads, hd, qs, ks, cs, sn, res,
        reinterpret_cast<const int4*>(h_coords), fwd, 0);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_qknorm_rope2d(void* qkv, int64_t l, int32_t heads, int32_t hd, const float* qs, const float* ks,
                                  const float* cs, const float* sn, int32_t n_prefix, vdit_stream_t stream) {
    if (l < 0 || heads < 1 || hd < 4 || hd % 8 || !qkv || !qs || !ks || n_prefix < 0) return VDIT_ERR_ARG;
    if (l > n_prefix && (!cs || !sn)) return VDIT_ERR_ARG;
    if (!aligned16(qkv)) return VDIT_ERR_ALIGN;
    if (l == 0) return VDIT_OK;
    if (hd > 128) return VDIT_ERR_UNSUPPORTED;
    qknorm_rope_kernel<1><<<blocks_for(l, kQkWarps), kQkWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(qkv), l, heads, hd, qs, ks, cs, sn, 1,
        nullptr, nullptr, n_prefix);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_vec_ln_modulate(const float* v, int32_t d, const float* s1, const float* sh, void* out,
                                    vdit_stream_t stream) {
    if (d <= 0 || !v || !s1 || !sh || !out) return VDIT_ERR_ARG;
    if (d > 2048) return VDIT_ERR_UNSUPPORTED;
    vec_ln_modulate_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(v, d, s1, sh,
                                                                            static_cast<__nv_bfloat16*>(out));
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_vec_gate_residual(float* c, const void* y, const float* g, int32_t d, vdit_stream_t stream) {
    if (d <= 0 || !c || !y || !g) return VDIT_ERR_ARG;
    vec_gate_residual_kernel<<<(d + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        c, static_cast<const __nv_bfloat16*>(y), g, d);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_swiglu_packed(const void* h, int64_t m, int32_t f, void* out, vdit_stream_t stream) {
    if (m < 0 || f <= 0 || f % 8 || !h || !out) return VDIT_ERR_ARG;
    if (!aligned16(h) || !aligned16(out)) return VDIT_ERR_ALIGN;
    if (m == 0) return VDIT_OK;
    swiglu_kernel<<<blocks_for(m * (f / 8), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(h), m, f, static_cast<__nv_bfloat16*>(out));
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_gather_rows_f32(const float* src, const int64_t* idx, int64_t n, int32_t c, float* dst,
                                    vdit_stream_t stream) {
    if (n < 0 || c <= 0 || !src || !idx || !dst) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    gather_rows_f32_kernel<<<blocks_for(n * c, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(src, idx, n, c, dst);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_cfg_euler(float* xt, const float* vp, const float* vn, int64_t n, float g, float dt,
                              vdit_stream_t stream) {
    if (n < 0 || !xt || !vp) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    cfg_euler_kernel<<<blocks_for(n * 16, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(xt, vp, vn, n * 16, g, dt);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_unpermute_denorm(const float* xt, const int64_t* up, int64_t n, const float* sc, const float* shf,
                                     float* out, vdit_stream_t stream) {
    if (n < 0 || !xt || !up || !sc || !shf || !out) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    unpermute_denorm_kernel<<<blocks_for(n * 16, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(xt, up, n, sc, shf, out);
    count_launches(1);
    return check_launch();
}
