/*
 * vdit.h -- C ABI of the B200 (sm_100a) sparse-voxel DiT (lat_dit) forward path.
 *
 * Conventions
 *  - Every entry point returns VDIT_OK (0) or a negative VDIT_ERR_* code and
 *    never throws.  Shapes are checked on the host before any launch.
 *  - The caller owns every buffer: inputs, outputs and workspaces are device
 *    pointers allocated by the caller; the library keeps no pointer past
 *    return.  "bf16" buffers are IEEE bfloat16, row-major, contiguous along
 *    the last dimension; strides are in elements.
 *  - All work is enqueued on `stream` (a cudaStream_t passed as void*); calls
 *    are asynchronous and reentrant.
 *  - Citations name the reference interface each entry point replaces
 *    (paths relative to the reference project; BK/ = baseline_repo/3dgen-main/).
 */
#ifndef VDIT_H_
#define VDIT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* vdit_stream_t;

#define VDIT_OK 0
#define VDIT_ERR_ARG (-1)          /* bad shape / size / null pointer        */
#define VDIT_ERR_ALIGN (-2)        /* pointer or stride not 16-byte aligned  */
#define VDIT_ERR_LAUNCH (-3)       /* CUDA launch error                      */
#define VDIT_ERR_UNSUPPORTED (-4)  /* head_dim / width not supported         */
#define VDIT_ERR_WORKSPACE (-5)    /* workspace too small                    */
#define VDIT_ERR_DRIVER (-6)       /* driver entry point (tensor maps) failed */
#define VDIT_ERR_TOO_LARGE (-7)    /* beyond the fixed scratch of a no-alloc entry point */

/* ------------------------------------------------------------------ runtime */
const char* vdit_version(void);
const char* vdit_error_string(int code);
/* Name and message of the last CUDA error an entry point of this thread saw
 * ("" when none). */
const char* vdit_last_cuda_error(void);
/* Number of kernels this library has launched since load (all devices). */
long long vdit_launch_count(void);
/* Device error word of the current device (a bounded wait that ran out or an
 * index out of range seen by a kernel).  Synchronizes the device; clear!=0
 * resets the word.  Returns 0 when no error was recorded. */
int vdit_device_error(int clear);

/* ------------------------------------------------------------------ geometry */
/* Workspace (bytes) for vdit_lex_perm / vdit_hilbert4_orders on n voxels. */
size_t vdit_geometry_workspace_bytes(int64_t n);

/* SparseDownsample(patch=1) order of one sample.  Replaces the key/argsort
 * block of _prepare_sample_geometry (lib/fast_flow.py:667-694) and
 * BK/base_models/sparse.py:998-1036.  vox [n,3] int32 (0 <= c < 1024, unique);
 * writes perm [n] int64, up_widx [n] int64 (inverse) and h_coords [n,4]
 * int32 = (0, vox[perm]). */
int vdit_lex_perm(const int32_t* vox, int64_t n, int64_t* perm, int64_t* up_widx,
                  int32_t* h_coords, void* workspace, size_t workspace_bytes,
                  vdit_stream_t stream);

/* Four Hilbert window orders (h, ht1, h1, ht) of one sample.  Replaces
 * _encode_hilbert_4_kernel + argsort in build_order_caches_fast
 * (lib/fast_kernels.py:1126-1154, 1792-1822; semantics BK/base_models/order.py:6-111).
 * h_coords [n,4] int32; coord_bound = exclusive upper bound of x,y,z (res).
 * Writes codes4 [4,n] int64 (may be NULL), fwd4 [4,n] int64, bwd4 [4,n] int64. */
int vdit_hilbert4_orders(const int32_t* h_coords, int64_t n, int32_t coord_bound,
                         int64_t* codes4, int64_t* fwd4, int64_t* bwd4,
                         void* workspace, size_t workspace_bytes, vdit_stream_t stream);

/* 27-neighbour submanifold index table.  Replaces libsparse.conv_indices
 * (BK/ops/libsparse/libsparse.cpp:29-37, conv.cu:21-163).  h_coords [n,4]
 * int32 must be sorted lexicographically by (b,x,y,z) (the output of
 * vdit_lex_perm); writes out [n,27] int32, -1 where the neighbour is absent. */
int vdit_conv_indices(const int32_t* h_coords, int64_t n, int32_t* out, vdit_stream_t stream);

/* RoPE tables in fp64 rounded to fp32.  Replace precompute_rope_3d_table /
 * precompute_rope_2d_cond (lib/fast_kernels.py:977-1035).
 * 3D: cos/sin [res, head_dim/6].  2D: cos/sin [cond_size^2, 2, head_dim/4]. */
int vdit_rope3d_table(int32_t res, int32_t head_dim, double base, float* cos_out, float* sin_out,
                      vdit_stream_t stream);
int vdit_rope2d_table(int32_t cond_size, int32_t head_dim, double base, float* cos_out,
                      float* sin_out, vdit_stream_t stream);

/* ------------------------------------------------------------------ row kernels */
/* x[n,d] bf16 = xt[n,16] fp32 @ w[d,16]^T (patchify, lib/fast_flow.py:931-935); xt, w, x 16-byte
 * aligned, d % 8 == 0, n < 2^31 (else VDIT_ERR_UNSUPPORTED). */
int vdit_patchify(const float* xt, int64_t n, const float* w, int32_t d, void* x_out,
                  vdit_stream_t stream);

/* out = LN(x) * scale1 + shift with scale1 = 1 + scale (fast_modulate,
 * lib/fast_kernels.py:672-885; BK/models/generators/lat_dit.py:63-66).
 * x, out bf16 [m,d]; scale1, shift fp32 [d]; d % 8 == 0, d <= 2048. */
int vdit_modulate(const void* x, int64_t m, int32_t d, const float* scale1, const float* shift,
                  void* out, vdit_stream_t stream);

/* x <- x + h * gate (in place, bf16) and, when mod_out != NULL,
 * mod_out = LN(x) * scale1 + shift.  h_row_stride 0 broadcasts one row of h.
 * Replaces _fused_gate_add_ln_modulate_kernel (lib/fast_kernels.py:556-611). */
int vdit_gate_add_modulate(void* x, const void* h, int64_t h_row_stride, int64_t m, int32_t d,
                           const float* gate, const float* scale1, const float* shift,
                           void* mod_out, vdit_stream_t stream);

/* Two gated residuals in one pass: x <- bf16(bf16(x + h * gate) + c2 * gate2), with c2
 * bf16 [d] one row broadcast to all rows, then (mod_out != NULL) the LayerNorm
 * modulation.  The 1-token branch's self-attention gate-add followed by its constant
 * cross-attention gate-add (BK/models/generators/lat_dit.py:345,473; lib/fast_flow.py:
 * 2295-2309), rounded as the two separate passes round. */
int vdit_gate_add2_modulate(void* x, const void* h, int64_t h_row_stride, int64_t m, int32_t d,
                            const float* gate, const void* c2, const float* gate2, const float* scale1,
                            const float* shift, void* mod_out, vdit_stream_t stream);

/* out[m,16] fp32 = bf16(LN(x) * scale1 + shift) @ w[16,d]^T.  Replaces
 * _fused_out_modulate_unpatchify_kernel (lib/fast_kernels.py:613-648, 888-940). */
int vdit_out_modulate_unpatchify(const void* x, int64_t m, int32_t d, const float* scale1,
                                 const float* shift, const float* w, float* out,
                                 vdit_stream_t stream);

/* The unpatchify projection alone, for rows already modulated (the last block's fused gate-add +
 * LayerNorm + AdaLN with the output modulation): out[m,16] fp32 = y[m,d] (bf16) @ w[16,d]^T at
 * fp32 accuracy on the tensor cores, w given as its three-part bf16 split w3 [48,d] from
 * vdit_split_weight3.  y, w3, out 16-byte aligned; d % 8 == 0; m < 2^31.  The projection of
 * lib/fast_kernels.py:613-648 (its fp32 weight, lib/fast_flow.py:144-148). */
int vdit_unpatchify_project(const void* y, int64_t m, int32_t d, const void* w3, float* out,
                            vdit_stream_t stream);

/* w3[3*rows, d] bf16 = the three-part split of w[rows, d] fp32: row p*rows + o holds part p of
 * row o, hi = bf16(w), mid = bf16(w - hi), lo = bf16(w - hi - mid) (hi + mid + lo = w to fp32
 * precision).  Made once per weight for vdit_unpatchify_project (rows = 16). */
int vdit_split_weight3(const float* w, int32_t rows, int32_t d, void* w3, vdit_stream_t stream);

/* out[j] = (RoPE3D(RMS(q[src])*q_scale), RoPE3D(RMS(k[src])*k_scale), v[src]),
 * src = fwd[j] (NULL: identity).  qkv/out bf16 [n,3,heads,head_dim];
 * q_scale/k_scale fp32 [heads,head_dim]; cos/sin fp32 [res, head_dim/6];
 * h_coords [n,4] int32 (coordinates of input rows, < res).  Replaces
 * _fused_qknorm_rope3d_gather_kernel (lib/fast_kernels.py:1156-1303, 1476-1535). */
int vdit_qknorm_rope3d_gather(const void* qkv, int64_t n, int32_t heads, int32_t head_dim,
                              const float* q_scale, const float* k_scale, const float* cos_t,
                              const float* sin_t, int32_t res, const int32_t* h_coords,
                              const int64_t* fwd, void* out, vdit_stream_t stream);

/* Context tokens, in place: q,k <- RMS(.)*scale, then 2D RoPE on tokens
 * >= n_prefix using cos/sin [l - n_prefix, 2, head_dim/4].  Replaces
 * _fused_qknorm_rope2d_cond_inplace_kernel (lib/fast_kernels.py:1305-1473). */
int vdit_qknorm_rope2d(void* qkv, int64_t l, int32_t heads, int32_t head_dim, const float* q_scale,
                       const float* k_scale, const float* cos2d, const float* sin2d,
                       int32_t n_prefix, vdit_stream_t stream);

/* Context-vector steps of the exact 1-token uncond branch (the reference runs them
 * as torch element-wise ops on the [D] fp32 context vector, lib/fast_flow.py:1702-1794,
 * 2295-2309).  vdit_vec_ln_modulate: out bf16 [d] = LN(v)*s1 + sh with eps 1e-6
 * (v fp32 [d], d <= 2048).  vdit_vec_gate_residual: c[d] fp32 += float(y[d] bf16) * g[d]. */
int vdit_vec_ln_modulate(const float* v, int32_t d, const float* s1, const float* sh, void* out,
                         vdit_stream_t stream);
int vdit_vec_gate_residual(float* c, const void* y, const float* g, int32_t d, vdit_stream_t stream);

/* Batched matrix-vector products for the one-row linears: the context vector of the exact
 * 1-token branch (the reference runs them as F.linear on a [1, D] row, lib/fast_flow.py:
 * 1142-1156, 1702-1794, 2295-2309) and the time-embedding / gate MLP (lib/fast_flow.py:
 * 455-654; BK/models/generators/lat_dit.py:631-635, 391-392, 409-410, 463-464, 817).
 *   out[b][r] = act(sum_i W[b][r][i] * x'[b][i] + bias[b][r]),  r < n, i < k, b < batch
 * x_mode selects the fused prologue that forms x' (fp32 accumulation throughout):
 *   VDIT_GEMV_X_BF16    x bf16 [k]
 *   VDIT_GEMV_X_F32     x fp32 [k]
 *   VDIT_GEMV_X_LN_MOD  x fp32 [k]: x' = bf16(LN(x) * mod_scale + mod_shift), eps 1e-6
 *   VDIT_GEMV_X_SWIGLU  x bf16 [2k] = [a | g]: x' = bf16(silu(g) * a)
 * W is bf16 (w_f32 = 0) or fp32 [n, k] per batch entry, 16-byte aligned, k a multiple of 8
 * (bf16) or 4 (fp32), k <= 8192; bias has W's type (or NULL).  out is bf16 or fp32 (out_f32)
 * [n] per entry, silu applied when silu_out.  Strides between batch entries are in elements
 * (x_bstride = 0 shares one input vector). */
#define VDIT_GEMV_X_BF16 0
#define VDIT_GEMV_X_F32 1
#define VDIT_GEMV_X_LN_MOD 2
#define VDIT_GEMV_X_SWIGLU 3
int vdit_gemv(int32_t x_mode, const void* x, int64_t x_bstride, const float* mod_scale,
              const float* mod_shift, int64_t mod_bstride, int32_t w_f32, const void* w,
              int64_t w_bstride, const void* bias, int64_t bias_bstride, int32_t out_f32,
              int32_t silu_out, void* out, int64_t out_bstride, int32_t n, int32_t k, int32_t batch,
              vdit_stream_t stream);

/* out[m,f] = silu(h[:, f:2f]) * h[:, :f] from packed h [m,2f] bf16.  Replaces
 * _fused_packed_swiglu_kernel (lib/fast_kernels.py:650-669, 942-974). */
int vdit_swiglu_packed(const void* h, int64_t m, int32_t f, void* out, vdit_stream_t stream);

/* Depthwise 27-tap submanifold conv: y[n,c] = b[c] + sum_d w[d,c] h[idx[n,d],c]
 * with fp32 weights/accumulation.  fuse_swiglu=0: out bf16 [n,c];
 * fuse_swiglu=1: out bf16 [n,c/2] = silu(y[:, c/2:]) * y[:, :c/2] with y
 * rounded to bf16 first.  Replaces libsparse.conv_fwd (BK/ops/libsparse/conv.cu:187-309,
 * libsparse.cpp:40-56) and, fused, the SwiGLU that follows it
 * (BK/models/generators/lat_dit.py:477-484). */
int vdit_dwconv27(const void* h, int64_t n, int32_t c, const int32_t* idx, const float* w,
                  const float* b, void* out, int32_t fuse_swiglu, vdit_stream_t stream);

/* The same conv with the SwiGLU fused, computed from a plan that stages each
 * block's neighbour rows in shared memory.  The plan plays the role of the
 * index table the reference builds once per voxel set and reuses in every
 * block and solver step (libsparse.conv_indices, BK/ops/libsparse/conv.cu:21-163,
 * consumed by conv_fwd, conv.cu:187-309): it is built from that table and a
 * space-filling-curve order of the rows (row_order [n] int64, a permutation of
 * [0,n), e.g. the Hilbert fwd order of vdit_hilbert4_orders) into a caller-owned
 * buffer of vdit_dwconv27_plan_bytes(n) bytes, and depends on nothing else.
 * The input h [n,c] bf16, weights w [27,c] and bias b [c] fp32 are given in
 * pair-interleaved column order: columns 4k..4k+3 hold (a[2k], a[2k+1],
 * gate[2k], gate[2k+1]) where the reference packs [a | gate]; a caller gets h in
 * this order by permuting the rows of the up-projection producing it.  out
 * [n,c/2] bf16 is in natural channel order and bit-identical to vdit_dwconv27
 * with fuse_swiglu=1 on the de-interleaved inputs.  c must be a multiple of 128
 * (VDIT_ERR_UNSUPPORTED otherwise); h, w, b and plan 16-byte aligned. */
size_t vdit_dwconv27_plan_bytes(int64_t n);
int vdit_dwconv27_plan(const int32_t* idx, const int64_t* row_order, int64_t n, void* plan,
                       size_t plan_bytes, vdit_stream_t stream);
int vdit_dwconv27_swiglu_planned(const void* h, int64_t n, int32_t c, const void* plan,
                                 const float* w, const float* b, void* out, vdit_stream_t stream);
/* The same conv + SwiGLU for weights w whose every value is exactly a bf16 value (as
 * when the reference upcasts a bf16 model's ffn_conv weight, lib/fast_flow.py:177):
 * its FMAs read the bf16 features and the bf16-rounded weights without unpacking them,
 * which is exact only under that precondition, and then the output is bit-identical to
 * vdit_dwconv27_swiglu_planned.  The precondition is the caller's to check (once per
 * weight set); the bias b has no such condition. */
int vdit_dwconv27_swiglu_planned_bf16w(const void* h, int64_t n, int32_t c, const void* plan,
                                       const float* w, const float* b, void* out, vdit_stream_t stream);

/* ------------------------------------------------------------------ attention */
/* Non-causal varlen flash attention on tcgen05 tensor cores (head_dim 96 or 128).
 * Row i of segment s attends to key rows [cu_k[s], cu_k[s+1]).  q/k/v point at
 * head 0 of row 0; row r head h lives at ptr + r*stride + h*head_dim (bf16).
 * out row for query row i is out_rows[i] when out_rows != NULL (scatter), else i.
 * cu_q_host/cu_k_host are HOST int32 arrays [nseg+1], nseg <= 128.
 * Replaces flash_attn varlen (qkv/kv packed) calls: sparse_windowed_sdp /
 * sparse_cross_sdp (BK/base_models/sparse.py:834-896), flash_varlen_qkvpacked_already_sorted,
 * flash_cond_self_attn, flash_cross_attn (lib/fast_kernels.py:1538-1646). */
int vdit_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                   int64_t v_stride, void* out, int64_t out_stride, const int64_t* out_rows,
                   const int32_t* cu_q_host, const int32_t* cu_k_host, int32_t nseg,
                   int32_t heads, int32_t head_dim, float softmax_scale, vdit_stream_t stream);

/* Workspace bytes for vdit_attention_1q over n_keys keys. */
size_t vdit_attention_1q_workspace_bytes(int32_t heads, int32_t head_dim, int64_t n_keys);

/* One query per head over n_keys keys (the exact 1-token uncond context->x
 * attention, lib/fast_flow.py:1769-1777).  q [heads,head_dim] bf16; k/v rows
 * at k + r*kv_stride + h*head_dim; out [heads,head_dim] bf16.  Split-K with
 * partials in the caller's workspace. */
int vdit_attention_1q(const void* q, const void* k, const void* v, int64_t kv_stride,
                      int64_t n_keys, int32_t heads, int32_t head_dim, float softmax_scale,
                      void* out, void* workspace, size_t workspace_bytes, vdit_stream_t stream);

/* Same computation as vdit_attention_1q, for callers that cannot allocate
 * device memory (an FFI host with no device allocator of its own, a serving loop
 * that must not touch the allocator between requests).  No
 * counterpart in the reference: it is an addition of this library.  The split-K
 * partials live in a fixed 1 MiB device array inside the library (one per GPU
 * that loads it, kept until process exit); heads * splits * (head_dim + 2) fp32
 * values must fit, else VDIT_ERR_TOO_LARGE (12 heads x 128 fits any n_keys).
 * The first call on a device, and the first call after that device's context was
 * re-created (a device reset), looks up the array's device address (make that call
 * before any stream capture).  Calls share the array: calls that overlap
 * on the GPU (different streams, or different threads on one device) race.
 * Allocates nothing; q, k, v, out as for vdit_attention_1q. */
int vdit_attention_1q_noalloc(const void* q, const void* k, const void* v, int64_t kv_stride,
                              int64_t n_keys, int32_t heads, int32_t head_dim, float softmax_scale,
                              void* out, vdit_stream_t stream);

/* The same single-query attention with the keys and values given as a linear of the
 * voxel rows, K = x wk^T + bk, V = x wv^T + bv (the 1-token branch's cross linear of
 * the modulated voxel stream, lib/fast_flow.py:1769-1777), without forming them: each
 * query is folded through wk, x is streamed once (fp32 scores, online softmax, the
 * probability-weighted sums of its rows), and wv, bv are applied to the merged sums
 * (bk shifts every score of a head equally and drops out).  q bf16 [heads*head_dim];
 * x bf16 [n, ldx]; wk, wv bf16 [heads*head_dim, ldw] (rows = output channels);
 * bv bf16 [heads*head_dim]; out bf16 [heads*head_dim].  heads <= 16,
 * heads*head_dim % 128 == 0 and <= 2048; workspace of
 * vdit_attention_1q_wide_workspace_bytes bytes. */
size_t vdit_attention_1q_wide_workspace_bytes(int32_t heads, int32_t head_dim, int64_t n_keys);
int vdit_attention_1q_wide(const void* q, const void* x, int64_t ldx, int64_t n, const void* wk, const void* wv,
                           int64_t ldw, const void* bv, int32_t heads, int32_t head_dim, float softmax_scale,
                           void* out, void* workspace, size_t workspace_bytes, vdit_stream_t stream);

/* ------------------------------------------------------------------ sparse conv (dense) */
/* Dense 27-tap sparse conv on tcgen05: out[n,co] = b[co] + sum_d sum_ci
 * W[d,co,ci] f[idx[n,d],ci].  f bf16 [n,cin]; w bf16 [27,cout,cin] (the
 * reference (3,3,3,cin,cout) weight transposed, as dense_conv_fwd_cuda does,
 * BK/ops/libsparse/conv.cu:601-645); b fp32 [cout]; out bf16 [n,cout].
 * cin % 64 == 0, cout % 256 == 0. */
int vdit_dense_conv27(const void* f, int64_t n, int32_t cin, int32_t cout, const int32_t* idx,
                      const void* w, const float* b, void* out, vdit_stream_t stream);

/* ------------------------------------------------------------------ block linears */
/* out[m,n] = bf16(sum_k a[m,k] w[n,k] + bias[n]) on tcgen05 (persistent CTA-pair
 * tiles of 256 rows x 256, 192 or 128 columns, fp32 accumulation in TMEM): the
 * nn.Linear of every block projection, BK/models/generators/lat_dit.py:306-345 (the
 * reference calls cuBLAS through F.linear with bf16 weights pre-cast,
 * lib/fast_flow.py:150-163).  a bf16 [m,lda], w bf16 [n,ldw], bias bf16 [n] or NULL,
 * out bf16 [m,ldo]; n and k multiples of 8 (a partial last column tile or k-step reads
 * zeros past n and k), leading dimensions multiples of 8, pointers 16-byte aligned. */
int vdit_linear(const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias, void* out,
                int64_t ldo, int64_t m, int32_t n, int32_t k, vdit_stream_t stream);

/* The self-attention to_qkv linear with the QK-norm / RoPE / window-order pass fused
 * into its epilogue: for input row r, out[dst_rows[r], :] = the three [heads, 128]
 * sections of bf16(a[r] . w^T + bias) with q and k replaced by
 * RoPE3D(bf16(RMSNorm(.)) * scale) at coords[r] = (b, x, y, z): the result of
 * vdit_linear followed by vdit_qknorm_rope3d_gather with fwd = the inverse of
 * dst_rows (lib/fast_flow.py:1450-1464, lib/fast_kernels.py:1476-1535).
 * head_dim 128 or 96 with an even number of heads (a CTA pair's tile holds two whole
 * heads); cos_t/sin_t [res, head_dim/6] fp32 (res <= 146 at 128, 192 at 96);
 * q_scale/k_scale [heads*head_dim] fp32; coords int32 [m, 4]; dst_rows int64 [m], a
 * permutation of 0..m-1. */
int vdit_linear_qkv_rope3d(const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias,
                           const float* q_scale, const float* k_scale, const float* cos_t, const float* sin_t,
                           int32_t res, const int32_t* coords, const int64_t* dst_rows, void* out, int64_t ldo,
                           int64_t m, int32_t heads, int32_t head_dim, int32_t k, vdit_stream_t stream);

/* ------------------------------------------------------------------ sampler glue */
/* dst[j,:] = src[idx[j],:] for fp32 rows of width c (noise[perm], lib/fast_flow.py:2576). */
int vdit_gather_rows_f32(const float* src, const int64_t* idx, int64_t n, int32_t c, float* dst,
                         vdit_stream_t stream);

/* CFG + Euler step on [n,16] fp32 (lib/fast_flow.py:2836,2887,3288):
 * v = v_pos + g*(v_pos - v_neg) (v_neg NULL: v = v_pos); xt -= dt * v. */
int vdit_cfg_euler(float* xt, const float* v_pos, const float* v_neg, int64_t n, float guidance,
                   float dt, vdit_stream_t stream);

/* Approximate CFG cache (opt-in; not part of the exact solver): one Euler step of a guided
 * step that skips the unconditional NFE and reuses the last unconditional velocity, the
 * reference's cfg_cache_mode "neg_reuse" (lib/fast_flow.py:2791-2887, non-QAOA branch).
 * With zero_star: nc = last_neg, blended toward the clean endpoint (1 - a) * last_neg +
 * a * (xt - last_neg_x0) / t_eval when last_neg_x0 is given and a = endpoint_blend > 0;
 * s = clamp(<vp, nc> / max(<nc, nc>, 1e-6), 0.9, 1.1); delta = vp - s * nc;
 * delta += hf_gain * (delta - row mean of delta).  Without it: delta = vp - last_neg.
 * Then xt -= dt * (vp + guidance * delta).  xt, vp, last_neg, last_neg_x0: [n, 16] fp32;
 * workspace of vdit_cfg_reuse_workspace_bytes() bytes (fixed-order reductions).
 * vdit_neg_endpoint: x0 = xt - t_eval * v_neg at a step that ran the unconditional NFE. */
size_t vdit_cfg_reuse_workspace_bytes(void);
int vdit_cfg_reuse_euler(float* xt, const float* vp, const float* last_neg, const float* last_neg_x0,
                         int64_t n, float guidance, float dt, float t_eval, float endpoint_blend,
                         float hf_gain, int32_t zero_star, void* workspace, size_t workspace_bytes,
                         vdit_stream_t stream);
int vdit_neg_endpoint(const float* xt, const float* v_neg, int64_t n, float t_eval, float* x0,
                      vdit_stream_t stream);

/* out[i,:] = xt[up_widx[i],:] * scale + shift, 16 channels (unpermute +
 * denormalize, lib/fast_flow.py:3306-3313). */
int vdit_unpermute_denorm(const float* xt, const int64_t* up_widx, int64_t n, const float* scale,
                          const float* shift, float* out, vdit_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* VDIT_H_ */
