// Single-query attention (one query per head over n keys): the context->x
// attention of the exact 1-token unconditional branch.  Pure streaming of
// K and V (2 * n * heads * head_dim bf16), so it is HBM-bound: split-K over
// many blocks, 16-byte loads, online softmax in fp32, partial states
// (max, sum, o[head_dim]) in the caller's workspace, then a combine kernel.
#include <cuda.h>
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace vdit {
namespace {

constexpr int kWarps = 4;
constexpr int kLanesPerKey = 16;     // 16 lanes x 8 bf16 = 128 channels (96 uses 12 lanes)
constexpr int kUnroll = 4;

__global__ void __launch_bounds__(kWarps * 32) attn1q_partial_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    int64_t kv_stride, int64_t n, int hd, float scale_log2, int splits, float* __restrict__ ws) {
    const int h = blockIdx.x, split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = lane / kLanesPerKey, vi = lane % kLanesPerKey;
    const bool active = vi * 8 < hd;
    const int64_t per = (n + splits - 1) / splits;
    const int64_t k0 = split * per, k1 = min(n, k0 + per);

    float qv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (active) {
        load8(q + (int64_t)h * hd + vi * 8, qv);
#pragma unroll
        for (int j = 0; j < 8; ++j) qv[j] *= scale_log2;
    }
    float m = -INFINITY, l = 0.f, o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int stride = kWarps * 2;          // keys per block step (2 slots per warp)
    // the loop bound is uniform across the warp (shuffles below need all 32 lanes)
    for (int64_t wbase = k0 + warp * 2; wbase < k1; wbase += (int64_t)stride * kUnroll) {
        const int64_t base = wbase + slot;
        float kv_[kUnroll][8], vv[kUnroll][8];
        bool ok[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t key = base + (int64_t)u * stride;
            ok[u] = key < k1;
            if (ok[u] && active) {
                load8_nc(k + key * kv_stride + (int64_t)h * hd + vi * 8, kv_[u]);
                load8_nc(v + key * kv_stride + (int64_t)h * hd + vi * 8, vv[u]);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) { kv_[u][j] = 0.f; vv[u][j] = 0.f; }
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) s = fmaf(qv[j], kv_[u][j], s);
#pragma unroll
            for (int off = kLanesPerKey / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            if (!ok[u]) continue;            // uniform within the 16-lane slot
            const float mn = fmaxf(m, s);
            const float a = exp2f(m - mn), p = exp2f(s - mn);
            l = l * a + p;
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = o[j] * a + p * vv[u][j];
            m = mn;
        }
    }
    // combine the 2*kWarps slot states of this block
    __shared__ float sm[kWarps * 2], sl[kWarps * 2];
    __shared__ float so[kWarps * 2][128];
    const int sid = warp * 2 + slot;
    if (vi == 0) { sm[sid] = m; sl[sid] = l; }
    if (active)
#pragma unroll
        for (int j = 0; j < 8; ++j) so[sid][vi * 8 + j] = o[j];
    __syncthreads();
    float* out = ws + ((int64_t)h * splits + split) * (2 + hd);
    if (threadIdx.x < hd) {
        float mm = -INFINITY;
        for (int i = 0; i < kWarps * 2; ++i) mm = fmaxf(mm, sm[i]);
        float acc = 0.f, ll = 0.f;
        for (int i = 0; i < kWarps * 2; ++i) {
            if (sm[i] == -INFINITY) continue;
            const float w = exp2f(sm[i] - mm);
            acc += so[i][threadIdx.x] * w;
            ll += sl[i] * w;
        }
        out[2 + threadIdx.x] = acc;
        if (threadIdx.x == 0) { out[0] = mm; out[1] = ll; }
    }
}

__global__ void attn1q_combine_kernel(const float* __restrict__ ws, int splits, int hd, __nv_bfloat16* __restrict__ out) {
    const int h = blockIdx.x, c = threadIdx.x;
    if (c >= hd) return;
    const float* base = ws + (int64_t)h * splits * (2 + hd);
    float mm = -INFINITY;
    for (int i = 0; i < splits; ++i) mm = fmaxf(mm, base[i * (2 + hd)]);
    float acc = 0.f, ll = 0.f;
    for (int i = 0; i < splits; ++i) {
        const float mi = base[i * (2 + hd)];
        if (mi == -INFINITY) continue;
        const float w = exp2f(mi - mm);
        ll += base[i * (2 + hd) + 1] * w;
        acc += base[i * (2 + hd) + 2 + c] * w;
    }
    out[(int64_t)h * hd + c] = f2bf(acc / ll);
}

int choose_splits(int heads, int64_t n) {
    int64_t target = (4 * 148 + heads - 1) / heads;       // ~4 blocks per SM
    int64_t by_len = (n + 127) / 128;                      // at least 128 keys per split
    int64_t s = target < by_len ? target : by_len;
    if (s < 1) s = 1;
    if (s > 4096) s = 4096;
    return (int)s;
}

}  // namespace
}  // namespace vdit

using namespace vdit;

extern "C" size_t vdit_attention_1q_workspace_bytes(int32_t heads, int32_t hd, int64_t n) {
    if (heads < 1 || hd < 1 || n < 1) return 0;
    return (size_t)heads * choose_splits(heads, n) * (2 + hd) * sizeof(float);
}

extern "C" int vdit_attention_1q(const void* q, const void* k, const void* v, int64_t kv_stride, int64_t n,
                                 int32_t heads, int32_t hd, float scale, void* out, void* ws, size_t ws_bytes,
                                 vdit_stream_t stream) {
    if (!q || !k || !v || !out || heads < 1 || n < 1 || kv_stride < (int64_t)heads * hd) return VDIT_ERR_ARG;
    if (hd % 8 || hd > 128) return VDIT_ERR_UNSUPPORTED;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (kv_stride % 8)) return VDIT_ERR_ALIGN;
    const int splits = choose_splits(heads, n);
    if (!ws || ws_bytes < (size_t)heads * splits * (2 + hd) * sizeof(float)) return VDIT_ERR_WORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float scale_log2 = scale * 1.4426950408889634f;
    attn1q_partial_kernel<<<dim3(heads, splits), kWarps * 32, 0, s>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
        kv_stride, n, hd, scale_log2, splits, static_cast<float*>(ws));
    attn1q_combine_kernel<<<heads, 128, 0, s>>>(static_cast<const float*>(ws), splits, hd, static_cast<__nv_bfloat16*>(out));
    count_launches(2);
    return check_launch();
}

// ---------------------------------------------------------------- allocation-free variant
// Some callers cannot allocate device memory at the point where they run this
// kernel: foreign-language hosts that reach the library through a plain FFI
// and have no device allocator of their own, and serving loops that must not
// touch the allocator between requests.
// For them vdit_attention_1q_noalloc keeps the split-K partials in a fixed
// file-scope device array instead of a caller workspace.  The array exists
// once per GPU that loads the library and lives until the process exits.
namespace vdit {
namespace {

constexpr size_t kNoAllocScratchFloats = 256 * 1024;   // 1 MiB of fp32 partials per device
__device__ __align__(256) float g_attn1q_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
struct ScratchEntry {
    CUcontext ctx;        // the context the address was looked up in
    float* addr;
};
ScratchEntry g_scratch[kMaxDevices] = {};

// The current driver context (null when the driver entry point is unavailable): a
// device reset or a context destroyed and re-created reloads the module, which moves
// the array, so a cached address is only valid in the context it was looked up in.
CUcontext current_context() {
    using Fn = CUresult (*)(CUcontext*);
    static Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(p);
    });
    CUcontext c = nullptr;
    if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
    return c;
}

// Device address of the scratch array on the current device, looked up once per device
// and context (the host-side symbol is not a device address and must not reach a kernel).
int scratch_address(float** addr) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        record_cuda_error(e);
        return VDIT_ERR_LAUNCH;
    }
    if (dev < 0 || dev >= kMaxDevices) return VDIT_ERR_UNSUPPORTED;
    const CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    ScratchEntry& ent = g_scratch[dev];
    if (ent.addr == nullptr || ctx == nullptr || ent.ctx != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn1q_scratch);
        if (e != cudaSuccess) {
            record_cuda_error(e);
            return VDIT_ERR_LAUNCH;
        }
        ent.addr = static_cast<float*>(p);
        ent.ctx = ctx;
    }
    *addr = ent.addr;
    return VDIT_OK;
}

}  // namespace
}  // namespace vdit

extern "C" int vdit_attention_1q_noalloc(const void* q, const void* k, const void* v, int64_t kv_stride, int64_t n,
                                         int32_t heads, int32_t hd, float scale, void* out, vdit_stream_t stream) {
    if (!q || !k || !v || !out || heads < 1 || n < 1 || kv_stride < (int64_t)heads * hd) return VDIT_ERR_ARG;
    if (hd % 8 || hd > 128) return VDIT_ERR_UNSUPPORTED;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (kv_stride % 8)) return VDIT_ERR_ALIGN;
    const int splits = choose_splits(heads, n);
    if ((size_t)heads * splits * (2 + hd) > kNoAllocScratchFloats) return VDIT_ERR_TOO_LARGE;
    float* ws = nullptr;
    const int rc = scratch_address(&ws);
    if (rc != VDIT_OK) return rc;
    // Every slot the combine kernel reads is written by the partial kernel of the
    // same call, so the array needs no clearing between calls.
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float scale_log2 = scale * 1.4426950408889634f;
    attn1q_partial_kernel<<<dim3(heads, splits), kWarps * 32, 0, s>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
        kv_stride, n, hd, scale_log2, splits, ws);
    attn1q_combine_kernel<<<heads, 128, 0, s>>>(ws, splits, hd, static_cast<__nv_bfloat16*>(out));
    count_launches(2);
    return check_launch();
}
