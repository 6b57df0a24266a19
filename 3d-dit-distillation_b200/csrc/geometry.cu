// Per-sample static geometry: lexicographic permutation, four Hilbert window
// orders, 27-neighbour conv_indices and RoPE tables.  Integer outputs are
// bit-exact with the reference (see oracle/geometry.py for the restatement).
#include <cub/device/device_radix_sort.cuh>
#include <math.h>

#include "common.cuh"

namespace vdit {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------- lex order
// key = x<<20 | y<<10 | z (lib/fast_flow.py:675-679); value = row index.
__global__ void lex_keys_kernel(const int32_t* __restrict__ vox, int64_t n,
                                uint64_t* __restrict__ keys, int64_t* __restrict__ iota) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint64_t x = (uint32_t)vox[3 * i], y = (uint32_t)vox[3 * i + 1], z = (uint32_t)vox[3 * i + 2];
    keys[i] = (x << 20) | (y << 10) | z;
    iota[i] = i;
}

__global__ void lex_finish_kernel(const int32_t* __restrict__ vox, const int64_t* __restrict__ perm,
                                  int64_t n, int64_t* __restrict__ up, int4* __restrict__ hc) {
    int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= n) return;
    int64_t src = perm[j];
    up[src] = j;
    hc[j] = make_int4(0, vox[3 * src], vox[3 * src + 1], vox[3 * src + 2]);
}

// ---------------------------------------------------------------- Hilbert
// 16-level 3D Hilbert distance (BK/base_models/order.py:6-53); the level loop
// always starts at bit 15 so the orientation matches for any coordinate range.
__device__ __forceinline__ uint64_t spread3(uint64_t w) {
    w &= 0x1FFFFFull;
    w = (w | (w << 32)) & 0x001F00000000FFFFull;
    w = (w | (w << 16)) & 0x001F0000FF0000FFull;
    w = (w | (w << 8)) & 0x010F00F00F00F00Full;
    w = (w | (w << 4)) & 0x10C30C30C30C30C3ull;
    w = (w | (w << 2)) & 0x1249249249249249ull;
    return w;
}

__device__ __forceinline__ uint64_t hilbert3(int64_t x, int64_t y, int64_t z) {
#pragma unroll
    for (int i = 15; i > 0; --i) {
        const int64_t q = 1ll << i, p = q - 1;
        if (x & q) x ^= p;
        int64_t t = (x ^ y) & p;
        if (y & q) { x ^= p; } else { x ^= t; y ^= t; }
        t = (x ^ z) & p;
        if (z & q) { x ^= p; } else { x ^= t; z ^= t; }
    }
    y ^= x;
    z ^= y;
    int64_t t = 0;
#pragma unroll
    for (int i = 15; i > 0; --i) {
        const int64_t q = 1ll << i;
        if (z & q) t ^= q - 1;
    }
    x ^= t; y ^= t; z ^= t;
    return (spread3((uint64_t)x) << 2) | (spread3((uint64_t)y) << 1) | spread3((uint64_t)z);
}

// codes of orders (h, ht1, h1, ht) = (x,y,z), (y+1,x+1,z+1), (x+1,y+1,z+1), (y,x,z)
// with the batch index at bit 48 (lib/fast_kernels.py:1126-1154).
__global__ void hilbert4_kernel(const int4* __restrict__ hc, int64_t n, uint64_t* __restrict__ codes,
                                int64_t* __restrict__ iota) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    int4 c = hc[i];
    uint64_t b = (uint64_t)(uint32_t)c.x << 48;
    codes[i] = hilbert3(c.y, c.z, c.w) | b;
    codes[n + i] = hilbert3(c.z + 1, c.y + 1, c.w + 1) | b;
    codes[2 * n + i] = hilbert3(c.y + 1, c.z + 1, c.w + 1) | b;
    codes[3 * n + i] = hilbert3(c.z, c.y, c.w) | b;
    iota[i] = i;
}

__global__ void inverse_perm_kernel(const int64_t* __restrict__ fwd, int64_t n, int64_t* __restrict__ bwd) {
    int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= n) return;
    bwd[fwd[j]] = j;
}

// ---------------------------------------------------------------- conv_indices
// key = b<<36 | x<<24 | y<<12 | z (BK/ops/libsparse/conv.cu:21-27); rows of
// h_coords are sorted by it, so a binary search over the rows returns the
// neighbour's row directly.  Search range narrowed to [key(min corner),
// key(max corner)] as in conv.cu:88-105.
__device__ __forceinline__ uint64_t conv_key(int b, int x, int y, int z) {
    return ((uint64_t)(uint32_t)b << 36) | ((uint64_t)(uint32_t)x << 24) |
           ((uint64_t)(uint32_t)y << 12) | (uint64_t)(uint32_t)z;
}

__device__ __forceinline__ uint64_t row_key(const int4* __restrict__ hc, int64_t r) {
    int4 c = __ldg(hc + r);
    return conv_key(c.x, c.y, c.z, c.w);
}

// last row index r in [lo, hi) with key(r) <= k, or lo-1 if none
__device__ __forceinline__ int64_t upper_le(const int4* __restrict__ hc, int64_t lo, int64_t hi, uint64_t k) {
    int64_t l = lo - 1, r = hi;   // invariant: key(l) <= k < key(r)
    while (r - l > 1) {
        int64_t m = (l + r) >> 1;
        if (row_key(hc, m) <= k) l = m; else r = m;
    }
    return l;
}

__global__ void conv_indices_kernel(const int4* __restrict__ hc, int64_t n, int32_t* __restrict__ out) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    int4 c = hc[i];
    const int lim = (1 << 12) - 1;
    uint64_t kmin = conv_key(c.x, max(c.y - 1, 0), max(c.z - 1, 0), max(c.w - 1, 0));
    uint64_t kmax = conv_key(c.x, min(c.y + 1, lim), min(c.z + 1, lim), min(c.w + 1, lim));
    int64_t lo = upper_le(hc, 0, n, kmin);
    if (lo < 0) lo = 0;
    int64_t hi = upper_le(hc, lo, n, kmax) + 1;
    int32_t* o = out + i * 27;
#pragma unroll 1
    for (int d = 0; d < 27; ++d) {
        int x = c.y + d / 9 - 1, y = c.z + (d / 3) % 3 - 1, z = c.w + d % 3 - 1;
        int32_t found = -1;
        if (d == 13) {
            found = (int32_t)i;
        } else if (x >= 0 && y >= 0 && z >= 0) {
            uint64_t k = conv_key(c.x, x, y, z);
            int64_t r = upper_le(hc, lo, hi, k);
            if (r >= lo && row_key(hc, r) == k) found = (int32_t)r;
        }
        o[d] = found;
    }
}

// ---------------------------------------------------------------- RoPE tables
__global__ void rope3d_table_kernel(int res, int m, double base, float* cs, float* sn) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= res * m) return;
    int r = i / m, f = i % m;
    double pos = ((double)r + 0.5) / (double)res * 2.0 - 1.0;
    double inv = pow(base, -(double)f / (double)m);
    double a = pos * inv;
    cs[i] = (float)cos(a);
    sn[i] = (float)sin(a);
}

__global__ void rope2d_table_kernel(int size, int m, double base, float* cs, float* sn) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    int total = size * size * 2 * m;
    if (i >= total) return;
    int f = i % m, ax = (i / m) % 2, tok = i / (2 * m);
    int coord = ax == 0 ? tok / size : tok % size;
    double pos = ((double)coord + 0.5) / (double)size * 2.0 - 1.0;
    double inv = pow(base, -(double)f / (double)m);
    double a = pos * inv;
    cs[i] = (float)cos(a);
    sn[i] = (float)sin(a);
}

inline unsigned grid_for(int64_t n) { return (unsigned)((n + kThreads - 1) / kThreads); }

int bit_length(uint64_t v) {
    int b = 0;
    while (v) { ++b; v >>= 1; }
    return b;
}

// CUB onesweep radix sort: histogram + exclusive-sum + one kernel per 8-bit pass
int sort_launches(int64_t n, int bits) {
    if (n <= 1) return 0;
    if (n <= 256 * 8) return 1;
    return 2 + (bits + 7) / 8;
}

struct SortBuffers {
    uint64_t* keys_in;
    uint64_t* keys_out;
    int64_t* vals_in;
    void* cub_tmp;
    size_t cub_bytes;
};

size_t cub_sort_bytes(int64_t n) {
    size_t bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, (const uint64_t*)nullptr, (uint64_t*)nullptr,
                                    (const int64_t*)nullptr, (int64_t*)nullptr, (int)n, 0, 64);
    return bytes;
}

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// workspace layout: keys_in[4n] | keys_out[n] | vals_in[n] | cub tmp
bool carve(void* ws, size_t ws_bytes, int64_t n, SortBuffers& sb) {
    size_t off = 0;
    char* base = static_cast<char*>(ws);
    sb.keys_in = reinterpret_cast<uint64_t*>(base + off);  off = align256(off + 4 * n * sizeof(uint64_t));
    sb.keys_out = reinterpret_cast<uint64_t*>(base + off); off = align256(off + n * sizeof(uint64_t));
    sb.vals_in = reinterpret_cast<int64_t*>(base + off);   off = align256(off + n * sizeof(int64_t));
    sb.cub_tmp = base + off;
    sb.cub_bytes = cub_sort_bytes(n);
    return off + sb.cub_bytes <= ws_bytes;
}

}  // namespace
}  // namespace vdit

using namespace vdit;

extern "C" size_t vdit_geometry_workspace_bytes(int64_t n) {
    if (n < 1) n = 1;
    return align256(4 * n * sizeof(uint64_t)) + align256(n * sizeof(uint64_t)) +
           align256(n * sizeof(int64_t)) + cub_sort_bytes(n) + 256;
}

extern "C" int vdit_lex_perm(const int32_t* vox, int64_t n, int64_t* perm, int64_t* up_widx,
                             int32_t* h_coords, void* ws, size_t ws_bytes, vdit_stream_t stream) {
    if (n < 0 || (n > 0 && (!vox || !perm || !up_widx || !h_coords))) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    if (n > INT32_MAX) return VDIT_ERR_ARG;
    if (!aligned16(h_coords)) return VDIT_ERR_ALIGN;
    SortBuffers sb;
    if (!ws || !carve(ws, ws_bytes, n, sb)) return VDIT_ERR_WORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    lex_keys_kernel<<<grid_for(n), kThreads, 0, s>>>(vox, n, sb.keys_in, sb.vals_in);
    size_t bytes = sb.cub_bytes;
    if (cub::DeviceRadixSort::SortPairs(sb.cub_tmp, bytes, sb.keys_in, sb.keys_out, sb.vals_in, perm,
                                        (int)n, 0, 30, s) != cudaSuccess)
        return VDIT_ERR_LAUNCH;
    lex_finish_kernel<<<grid_for(n), kThreads, 0, s>>>(vox, perm, n, up_widx, reinterpret_cast<int4*>(h_coords));
    count_launches(2 + sort_launches(n, 30));
    return check_launch();
}

extern "C" int vdit_hilbert4_orders(const int32_t* h_coords, int64_t n, int32_t coord_bound,
                                    int64_t* codes4, int64_t* fwd4, int64_t* bwd4, void* ws,
                                    size_t ws_bytes, vdit_stream_t stream) {
    if (n < 0 || coord_bound < 1 || coord_bound > 65535) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    if (!h_coords || !fwd4 || !bwd4 || n > INT32_MAX) return VDIT_ERR_ARG;
    if (!aligned16(h_coords)) return VDIT_ERR_ALIGN;
    SortBuffers sb;
    if (!ws || !carve(ws, ws_bytes, n, sb)) return VDIT_ERR_WORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint64_t* codes = codes4 ? reinterpret_cast<uint64_t*>(codes4) : sb.keys_in;
    hilbert4_kernel<<<grid_for(n), kThreads, 0, s>>>(reinterpret_cast<const int4*>(h_coords), n, codes, sb.vals_in);
    // shifted coordinates reach coord_bound; codes stay below 2^(3*bits) for batch 0.
    // Batch indices live at bit 48 and above; one sample has batch 0.
    int bits = 3 * bit_length((uint64_t)coord_bound);
    if (bits > 48) bits = 48;
    int launches = 1;
    for (int o = 0; o < 4; ++o) {
        size_t bytes = sb.cub_bytes;
        if (cub::DeviceRadixSort::SortPairs(sb.cub_tmp, bytes, codes + o * n, sb.keys_out, sb.vals_in,
                                            fwd4 + o * n, (int)n, 0, bits, s) != cudaSuccess)
            return VDIT_ERR_LAUNCH;
        inverse_perm_kernel<<<grid_for(n), kThreads, 0, s>>>(fwd4 + o * n, n, bwd4 + o * n);
        launches += 1 + sort_launches(n, bits);
    }
    count_launches(launches);
    return check_launch();
}

extern "C" int vdit_conv_indices(const int32_t* h_coords, int64_t n, int32_t* out, vdit_stream_t stream) {
    if (n < 0 || (n > 0 && (!h_coords || !out)) || n > INT32_MAX) return VDIT_ERR_ARG;
    if (n == 0) return VDIT_OK;
    if (!aligned16(h_coords)) return VDIT_ERR_ALIGN;
    conv_indices_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const int4*>(h_coords), n, out);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_rope3d_table(int32_t res, int32_t head_dim, double base, float* cs, float* sn,
                                 vdit_stream_t stream) {
    if (res < 1 || head_dim < 6 || !cs || !sn) return VDIT_ERR_ARG;
    int m = head_dim / 6;
    rope3d_table_kernel<<<grid_for((int64_t)res * m), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        res, m, base, cs, sn);
    count_launches(1);
    return check_launch();
}

extern "C" int vdit_rope2d_table(int32_t size, int32_t head_dim, double base, float* cs, float* sn,
                                 vdit_stream_t stream) {
    if (size < 1 || head_dim < 4 || !cs || !sn) return VDIT_ERR_ARG;
    int m = head_dim / 4;
    rope2d_table_kernel<<<grid_for((int64_t)size * size * 2 * m), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        size, m, base, cs, sn);
    count_launches(1);
    return check_launch();
}
