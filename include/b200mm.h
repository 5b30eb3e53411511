/*
 * b200mm.h -- C ABI of the B200 (sm_100a) matmul hot path of the llms Qwen3 engine.
 *
 * Every entry point takes device pointers, sizes and row strides (in ELEMENTS),
 * an opaque cudaStream_t (passed as void*), and returns an int status
 * (B200MM_OK == 0).  Nothing here allocates or frees device memory: outputs and
 * workspaces are owned by the caller (PyTorch's caching allocator in the Python
 * shim).  No entry point synchronises the stream, so every call can be issued
 * back to back and captured in a CUDA graph.
 *
 * Inner (column) strides are 1 for every matrix: the caller makes a tensor
 * contiguous in its last dimension before the call.  Row strides may be larger
 * than the row length.  Shapes and dtypes are validated on the host before any
 * launch; an invalid call returns a status and launches nothing.
 *
 * Reference interfaces replaced (paths inside the aaholmes/llms project):
 *   b200mm_gate_up_silu      <- kernels/fused_ffn.py:98-152  triton_fused_gate_up_silu
 *                               (launch of _fused_gate_up_silu_kernel, fused_ffn.py:20-95)
 *   b200mm_qkv               <- kernels/fused_qkv.py:88-149  triton_fused_qkv
 *                               (launch of _qkv_matmul_kernel, fused_qkv.py:28-85)
 *   b200mm_gate_up_silu_w8   <- no reference symbol: int8 weight-only variant of
 *   b200mm_qkv_w8               the two calls above (dequantise W = q * s[row])
 *   b200mm_mla_append        <- engine/mla.py:211-242 for one token at a time: the
 *                               per-token k_norm factor of the reconstructed K head
 *                               and the RoPE'd rope half of K, kept as side-bands
 *   b200mm_mla_decode        <- engine/mla.py:195-264, the T == 1 branch of
 *                               MLAttention.forward (everything between the
 *                               q/dkv/kr projections and the o projection)
 *   b200mm_rmsnorm           <- engine/attention.py:20-33 RMSNorm.forward, with the
 *                               residual add of engine/model.py:54-63 folded in
 *   b200mm_qk_norm_rope      <- engine/attention.py:119-131 (T == 1): q_norm,
 *                               k_norm, apply_rope and the KV-cache write
 */
#ifndef B200MM_H_
#define B200MM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200MM_ABI_VERSION 2

/* status codes */
enum {
  B200MM_OK = 0,
  B200MM_ERR_SHAPE = 1,        /* a size is <= 0, too large, or inconsistent */
  B200MM_ERR_ALIGN = 2,        /* pointer / stride alignment the kernel needs */
  B200MM_ERR_DTYPE = 3,        /* unsupported dtype code */
  B200MM_ERR_LAUNCH = 4,       /* cudaGetLastError() after the launch */
  B200MM_ERR_ARG = 5,          /* null pointer or bad scalar argument */
  B200MM_ERR_WORKSPACE = 6,    /* workspace pointer null or too small */
  B200MM_ERR_DEVICE = 7,       /* device is not sm_100 or a runtime query failed */
  B200MM_ERR_TIMEOUT = 8       /* a bounded on-device wait gave up */
};

/* dtype codes for activations / dense weights / outputs */
enum {
  B200MM_F32 = 0,
  B200MM_F16 = 1,
  B200MM_BF16 = 2
};

/* Human-readable text for a status code (static storage, never NULL). */
const char* b200mm_status_string(int status);

/* B200MM_ABI_VERSION of the built library. */
int b200mm_abi_version(void);

/* Number of device kernels this library has launched since load (all
 * entry points, all devices).  Host-side counter; used by the bench to
 * report how many of its own kernels ran in a timed region. */
uint64_t b200mm_launch_count(void);

/*
 * Kernel-family override for cross-checking in tests:
 *   0 = automatic choice (default), 1 = always the generic kernels (the tiled
 *   CUDA-core projection and the generic MLA split kernel).
 * Process-wide; returns the previous value.  No reference counterpart.
 */
int b200mm_force_generic(int on);

/*
 * y[m, n] = silu(sum_k x[m,k] * wg[n,k]) * (sum_k x[m,k] * wu[n,k])
 *
 *   x  : [M, K]  dtype,  row stride ldx
 *   wg : [N, K]  dtype,  row stride ldwg   (nn.Linear weight layout (out, in))
 *   wu : [N, K]  dtype,  row stride ldwu
 *   y  : [M, N]  dtype,  row stride ldy
 * fp32 accumulation; silu(g) = g * sigmoid(g) on the fp32 accumulator; one
 * rounding to dtype on store.  Replaces kernels/fused_ffn.py:98-152.
 */
int b200mm_gate_up_silu(const void* x, int64_t ldx,
                        const void* wg, int64_t ldwg,
                        const void* wu, int64_t ldwu,
                        void* y, int64_t ldy,
                        int64_t M, int64_t N, int64_t K,
                        int dtype, void* stream);

/*
 * y[m, n] = sum_k x[m,k] * w[n,k]   with w = [Wq; Wk; Wv] row-stacked
 *
 *   x : [M, K], w : [N, K] (N = n_q + 2 n_k), y : [M, N]; all `dtype`.
 * The caller splits y's columns into q / k / v views.  Replaces
 * kernels/fused_qkv.py:88-149.
 */
int b200mm_qkv(const void* x, int64_t ldx,
               const void* w, int64_t ldw,
               void* y, int64_t ldy,
               int64_t M, int64_t N, int64_t K,
               int dtype, void* stream);

/*
 * Int8 weight-only variants (no reference counterpart; new in this build).
 *   wq : int8 [N, K] row stride ldw, values in [-127, 127]
 *   s  : fp32 [N]   per-output-channel scale, W[n,k] = wq[n,k] * s[n]
 *   x, y : `dtype` (F16 or BF16)
 * y = (x . wq^T) * s, accumulated in fp32; the gate/up variant applies
 * silu(g * sg) * (u * su).
 */
int b200mm_gate_up_silu_w8(const void* x, int64_t ldx,
                           const int8_t* wg, const float* sg,
                           const int8_t* wu, const float* su,
                           int64_t ldw,
                           void* y, int64_t ldy,
                           int64_t M, int64_t N, int64_t K,
                           int dtype, void* stream);

int b200mm_qkv_w8(const void* x, int64_t ldx,
                  const int8_t* w, const float* s, int64_t ldw,
                  void* y, int64_t ldy,
                  int64_t M, int64_t N, int64_t K,
                  int dtype, void* stream);

/*
 * Plain bias-free projection, y[m, n] = sum_k x[m,k] * w[n,k], on the same
 * kernel families as b200mm_qkv (decode GEMV, small-batch tensor-core GEMV,
 * tcgen05 GEMM).  Replaces the attention output projection `self.o(attn)`
 * (src/engine/attention.py:163) and the FFN down projection
 * `self.down(...)` (src/engine/model.py:37), both nn.Linear(bias=False).
 *   x : [M, K], w : [N, K], y : [M, N]; all `dtype`.
 */
int b200mm_linear(const void* x, int64_t ldx,
                  const void* w, int64_t ldw,
                  void* y, int64_t ldy,
                  int64_t M, int64_t N, int64_t K,
                  int dtype, void* stream);

/* Int8 weight-only b200mm_linear: y = (x . wq^T) * s (see the _w8 block above). */
int b200mm_linear_w8(const void* x, int64_t ldx,
                     const int8_t* w, const float* s, int64_t ldw,
                     void* y, int64_t ldy,
                     int64_t M, int64_t N, int64_t K,
                     int dtype, void* stream);

/*
 * GQA single-query decode attention over the engine's KV cache:
 *   out[b, h, :] = softmax_t(q[b, h, :] . k[b, h / g, t, :] * scale) v[b, h / g, t, :]
 * for t < L, g = H / KV.  This is what the engine's swappable decode op
 * computes (`Attention.decode_attn_op`, src/engine/attention.py:101-105 and
 * :138-145, which hands it the pre-expansion K/V views), and what its default
 * path (repeat_interleave + scaled_dot_product_attention,
 * src/engine/attention.py:147-150) computes for T == 1.
 *   q   : [B, H, D]  strides (q_sb, q_sh, 1)          `dtype`
 *   k, v: [B, KV, L, D] strides (sb, sh, st, 1)         `dtype`
 *   out : [B, H, D]  strides (o_sb, o_sh, 1)          `dtype`
 * Strides are in elements.  fp32 softmax and accumulation; one rounding on
 * store.  16-bit caches with D = 64 or 128, g <= 16 and contiguous token
 * rows (st == D) take the split-context kernel; everything else a generic
 * kernel.
 *   workspace: >= b200mm_gqa_decode_workspace_size(B, H, KV, D, L) bytes,
 *              256-byte aligned, owned by the stream until the call completes,
 *              ZERO-FILLED before its first use; every call leaves the few
 *              words it needs zeroed for the next call (no per-call memset).
 */
size_t b200mm_gqa_decode_workspace_size(int64_t B, int64_t H, int64_t KV, int64_t D, int64_t L);

int b200mm_gqa_decode(const void* q, int64_t q_sb, int64_t q_sh,
                      const void* k, int64_t k_sb, int64_t k_sh, int64_t k_st,
                      const void* v, int64_t v_sb, int64_t v_sh, int64_t v_st,
                      void* out, int64_t o_sb, int64_t o_sh,
                      int64_t B, int64_t H, int64_t KV, int64_t D, int64_t L,
                      float scale, int dtype,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * MLA latent-cache shapes shared by the two MLA entry points.
 *   B      batch rows served by this call (rows 0..B-1 of the cache)
 *   H      query heads, KV key/value groups (H % KV == 0)
 *   D      head_dim, DR = d_rope (last DR dims of a head carry RoPE),
 *          DN = D - DR
 *   R      latent rank
 * Cache tensors (engine/mla.py:41-87, MLAKVCache):
 *   c_kv       [*, S, R]       dtype, strides (c_sb, c_st) elements, unit inner
 *   k_rope_pre [*, S, KV, DR]  dtype, strides (r_sb, r_st), inner [KV, DR] dense
 *   (b200mm_mla_append reads k_rope_pre; the decode step reads its side-band kz)
 *   kscale     [*, S, KV]      fp32,  strides (s_sb, s_st), inner dense
 * Weights (the nn.Linear weights viewed per group):
 *   w_uk : [KV, DN, R] dtype dense (uk_nope.weight.view(KV, DN, R))
 *   w_uv : [KV, D, R]  dtype dense (uv.weight.view(KV, D, R))
 *   k_norm_w : fp32 [D]  (k_norm.weight)
 */
typedef struct b200mm_mla_shape {
  int32_t B, H, KV, D, DR, R;
  int32_t dtype;          /* B200MM_BF16 / F16 / F32 for cache, q, weights, out */
  float eps;              /* k_norm eps */
} b200mm_mla_shape;

/*
 * Per-token side-bands of the MLA cache, written once when tokens enter the
 * cache (positions [t0, t1) of batch rows 0..B-1), so a decode step never
 * re-expands or re-rotates K:
 *   kscale[b,t,g] fp32  = rsqrt(mean_d k[b,t,g,d]^2 + eps), where
 *                         k[b,t,g] = [w_uk[g] . c_kv[b,t] ; k_rope_pre[b,t,g]]
 *                         is the reconstructed, un-normed K head of
 *                         engine/mla.py:212-215; k_norm (engine/mla.py:221,
 *                         engine/attention.py:28-33) multiplies by it;
 *   kz[b,t,g,:]  dtype  = rope_t(k_norm_w[DN:] * k_rope_pre[b,t,g,:]), the RoPE
 *                         half of the normed K head divided by kscale
 *                         (engine/mla.py:226-242; angle float(t) * inv_freq[i],
 *                         rotate-half convention).
 *   kz : [*, S, KV, DR] dtype, strides (z_sb, z_st), inner [KV, DR] dense.
 */
int b200mm_mla_append(const b200mm_mla_shape* shape,
                      const void* c_kv, int64_t c_sb, int64_t c_st,
                      const void* k_rope_pre, int64_t r_sb, int64_t r_st,
                      const void* w_uk, const float* k_norm_w, const float* rope_inv_freq,
                      float* kscale, int64_t s_sb, int64_t s_st,
                      void* kz, int64_t z_sb, int64_t z_st,
                      int64_t t0, int64_t t1, void* stream);

/*
 * Bytes of workspace b200mm_mla_decode needs for (shape, L).  0 on bad shape.
 */
size_t b200mm_mla_decode_workspace_size(const b200mm_mla_shape* shape, int64_t L);

/*
 * One decode step of MLA attention with absorbed up-projections.
 *   q   : [B, H, D] dtype, batch stride q_sb (q after q_norm, before RoPE)
 *   kz, kscale : the side-bands of b200mm_mla_append, valid for positions < L
 *   L   : context length including the new token; the query sits at
 *         position L-1 and attends to cache positions 0..L-1
 *   rope_inv_freq : fp32 [DR/2]; angle(t, i) = float(t) * inv_freq[i]
 *   scale : softmax scale (head_dim ** -0.5 in the reference SDPA)
 *   out : [B, H, D] dtype, batch stride o_sb -- equals the SDPA output of
 *         engine/mla.py:262 transposed to (B, 1, H, D), i.e. the input of
 *         the o projection.
 *   workspace : >= b200mm_mla_decode_workspace_size(shape, L) bytes,
 *         256-byte aligned; contents need not be initialised.
 */
int b200mm_mla_decode(const b200mm_mla_shape* shape,
                      const void* q, int64_t q_sb,
                      const void* c_kv, int64_t c_sb, int64_t c_st,
                      const void* kz, int64_t z_sb, int64_t z_st,
                      const float* kscale, int64_t s_sb, int64_t s_st,
                      const void* w_uk, const void* w_uv,
                      const float* k_norm_w, const float* rope_inv_freq,
                      float scale, int64_t L,
                      void* out, int64_t o_sb,
                      void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * The MLA decode split over the context, for a step spread across GPUs when
 * the batch has fewer rows than GPUs (each GPU streams a slice of every row's
 * cache; the slices' partial softmaxes are merged afterwards).  Same math as
 * b200mm_mla_decode (engine/mla.py:195-264), cut in two:
 *
 * b200mm_mla_decode_partial: tokens [t_begin, t_end) of rows 0..B-1 for a
 *   query at position L - 1 (the RoPE of the query uses L; the pointers are
 *   the whole cache's).  Writes av_out fp32 [B, H, R] -- sum_t p_t c_t with p
 *   the softmax over the range -- and ml_out fp32 [B, H, 2] -- the range's
 *   (max score, sum of exp).  No W_uv step.  Workspace as
 *   b200mm_mla_decode_workspace_size(shape, t_end - t_begin).
 * b200mm_mla_combine_partials: nparts ranges' partials -- range r's av
 *   [B, H, R] at av_parts + r * av_part_stride and its ml [B, H, 2] at
 *   ml_parts + r * ml_part_stride (elements; nparts <= 64; so one gathered
 *   buffer per rank can hold both) -> out [B, H, D] =
 *   W_uv . (sum_r s_r e^(m_r - M) av_r / sum_r s_r e^(m_r - M)).  Workspace as
 *   b200mm_mla_decode_workspace_size(shape, 1).
 * No reference counterpart of the split itself: the reference runs one GPU.
 */
int b200mm_mla_decode_partial(const b200mm_mla_shape* shape,
                              const void* q, int64_t q_sb,
                              const void* c_kv, int64_t c_sb, int64_t c_st,
                              const void* kz, int64_t z_sb, int64_t z_st,
                              const float* kscale, int64_t s_sb, int64_t s_st,
                              const void* w_uk,
                              const float* k_norm_w, const float* rope_inv_freq,
                              float scale, int64_t L, int64_t t_begin, int64_t t_end,
                              float* av_out, float* ml_out,
                              void* workspace, size_t workspace_bytes,
                              void* stream);

int b200mm_mla_combine_partials(const b200mm_mla_shape* shape,
                                const float* av_parts, int64_t av_part_stride,
                                const float* ml_parts, int64_t ml_part_stride, int64_t nparts,
                                const void* w_uv,
                                void* out, int64_t o_sb,
                                void* workspace, size_t workspace_bytes,
                                void* stream);

/*
 * RMSNorm with the engine's rounding (src/engine/attention.py:20-33):
 *   y[m, :] = weight * cast(x32 * rsqrt(mean(x32^2) + eps)),  x32 = float(h[m, :])
 * on h = x, or, when `residual` is given, on h = cast(x + residual) -- the
 * residual add that precedes every norm of a decoder block
 * (src/engine/model.py:54-63: h = x + attn(norm1(x)); norm2(h)); h is then also
 * stored to `h_out` when it is not NULL.  x, residual, weight, h_out and y share
 * `dtype`; rows are 16-byte aligned; N <= 16384.  One launch replaces the
 * engine's chain of elementwise kernels (cast, pow, mean, rsqrt, mul, cast,
 * mul, and the add).
 */
int b200mm_rmsnorm(const void* x, int64_t ldx,
                   const void* residual, int64_t ldr,
                   void* h_out, int64_t ldh,
                   const void* weight,
                   void* y, int64_t ldy,
                   int64_t M, int64_t N, float eps,
                   int dtype, void* stream);

/*
 * QK-norm, RoPE and the KV-cache write of one new token per row
 * (src/engine/attention.py:119-131 for T == 1), straight from the fused QKV
 * projection's output qkv[b, :] = [q heads | k heads | v heads] (H, KV, KV
 * heads of D):
 *   q_out[b, h, :]          = rope(q_norm(q[b, h, :]), pos)
 *   k_cache[b, kh, pos, :]  = rope(k_norm(k[b, kh, :]), pos)
 *   v_cache[b, kh, pos, :]  = v[b, kh, :]
 * with the engine's rounding: the norms as b200mm_rmsnorm over D, RoPE as
 * x * cos + rotate_half(x) * sin in `dtype` (apply_rope, attention.py:59-72),
 * each product and the sum rounded to `dtype`; the cos / sin tables
 * [max_pos, D] are in `dtype` (the engine's model casts its tables with the
 * module).  The position is `pos`, or *pos_dev when pos_dev is not NULL (a
 * device scalar, for one CUDA graph replayed at every position; the caller
 * keeps it inside [0, max_pos)).  D is 64, 128 or 256.
 */
int b200mm_qk_norm_rope(const void* qkv, int64_t ldq,
                        int64_t B, int64_t H, int64_t KV, int64_t D,
                        const void* q_norm_w, const void* k_norm_w,
                        const void* cos_table, const void* sin_table, int64_t max_pos,
                        int64_t pos, const int64_t* pos_dev,
                        void* q_out, int64_t q_sb, int64_t q_sh,
                        void* k_cache, int64_t k_sb, int64_t k_sh, int64_t k_st,
                        void* v_cache, int64_t v_sb, int64_t v_sh, int64_t v_st,
                        float eps, int dtype, void* stream);

/*
 * b200mm_peer_gather -- stands in for the NCCL all-gather after each
 * column-sharded projection of the multi-GPU decode step (the reference
 * engine runs on one GPU; the gather is the only collective its sharded form
 * needs).  One launch: this rank's block src [rows, sum(part_widths)] is
 * stored into every rank's gathered buffer dst[r] [rows, ld_dst] over peer
 * memory, part j of rank q at column world * (w_0 + .. + w_{j-1}) + q * w_j,
 * so a fused QKV block [q | k | v] gathers to [all q | all k | all v].
 *   - dst[0..world) and flags[0..world) are device addresses valid on this
 *     GPU (peer mappings of every rank's buffers, own rank included);
 *     flags[r] is rank r's uint32 array [world][nctas], zeroed once before
 *     the first gather; seen is this rank's uint32 [nctas] (zeroed once),
 *     err a local int status word (zeroed once; set to 1 when a wait for a
 *     peer ran out, after 5 s, and then stays set).
 *   - Every rank must issue the same sequence of gathers with the same
 *     nctas; calls on one stream per rank.  Each CTA waits, bounded, for the
 *     peers' CTA of the same index, so when the kernel ends every rank's
 *     block has arrived.  A peer may write the next gather into dst before
 *     this rank has read the previous one unless each call site has its own
 *     dst region (or the reads finish before this rank's next gather).
 *   - dtype 0 / 1 / 2 (fp32 / fp16 / bf16); copies are 16 bytes wide when
 *     every address, width and stride allows.  world <= 8, nparts <= 3.
 */
int b200mm_peer_gather(const void* src, int64_t ld_src, int64_t rows,
                       const int64_t* part_widths, int nparts,
                       void* const* dst, int64_t ld_dst, int dtype,
                       int rank, int world, void* const* flags,
                       void* seen, void* err, int nctas, void* stream);

/*
 * Peer output of a projection (b200mm_*_peer): instead of a local y, the
 * projection stores its output columns straight into every rank's gathered
 * buffer, at the positions b200mm_peer_gather would give them; the launch's
 * last CTA counts the launch done on every peer, then waits,
 * bounded (5 s; *err = 1 when it runs out), until every peer's launch has
 * counted itself done here.
 *   dst[r], flags[r]: rank r's gathered buffer for this call site and its
 *     uint32 counter array [8] (zeroed once), as device addresses valid on
 *     this GPU; ld_dst: the gathered row stride (elements); part_widths /
 *     nparts: this rank's output columns as parts (the fused QKV: q, k, v);
 *   ticket, seen: this rank's uint32 words (zeroed once), err its status.
 * Every rank issues the same sequence of peer-output projections on one
 * stream, with the same shapes.
 */
typedef struct b200mm_peer_out {
  void* dst[8];
  int64_t ld_dst;
  int64_t part_widths[3];
  int32_t nparts;
  int32_t rank;
  int32_t world;
  int32_t reserved;
  void* flags[8];
  void* ticket;
  void* seen;
  void* err;
} b200mm_peer_out;

/*
 * b200mm_linear_peer, b200mm_linear_w8_peer, b200mm_gate_up_silu_w8_peer --
 * b200mm_linear / b200mm_linear_w8 / b200mm_gate_up_silu_w8 on this rank's
 * column shard, fused with the all-gather that follows them in the
 * column-sharded decode step (the compute step and the collective in one
 * kernel: the output tiles cross NVLink as they are produced).  Only the
 * decode regime runs fused -- M <= 8 for 16-bit weights (gate-up 16), M <= 32
 * for int8 -- other calls return B200MM_ERR_SHAPE and launch nothing (run
 * the projection into a local buffer and b200mm_peer_gather instead).
 */
int b200mm_linear_peer(const void* x, int64_t ldx, const void* w, int64_t ldw,
                       int64_t M, int64_t N, int64_t K, int dtype,
                       const b200mm_peer_out* out, void* stream);
int b200mm_linear_w8_peer(const void* x, int64_t ldx, const int8_t* w, const float* s, int64_t ldw,
                          int64_t M, int64_t N, int64_t K, int dtype,
                          const b200mm_peer_out* out, void* stream);
int b200mm_gate_up_silu_w8_peer(const void* x, int64_t ldx, const int8_t* wg, const float* sg,
                                const int8_t* wu, const float* su, int64_t ldw,
                                int64_t M, int64_t N, int64_t K, int dtype,
                                const b200mm_peer_out* out, void* stream);

/*
 * b200mm_mla_decode_noalloc -- no counterpart in the reference.
 *
 * b200mm_mla_decode for callers that cannot allocate device memory at decode
 * time (a server drawing on a fixed arena reserved at start-up, a replayed
 * CUDA graph whose allocations must not change, a plugin whose host framework
 * owns every allocation): same arguments minus the workspace, same kernels,
 * same results.  The workspace comes from one array compiled into the library
 * (8 MiB, 256-byte aligned; B = 32, L = 32768 at the Qwen3-4B MLA shape needs
 * about 7.8 MiB).  Every GPU that loads the library holds that array until the
 * process exits.
 *   - A call whose workspace would exceed 8 MiB returns B200MM_ERR_WORKSPACE
 *     and launches nothing (b200mm_mla_decode_workspace_size gives the need).
 *   - The first call on a device looks up the array's device address on that
 *     device (cudaGetSymbolAddress, the device current at the call); make that
 *     first call before any stream capture.  The looked-up address is kept
 *     for the life of the process: after cudaDeviceReset (or anything else
 *     that tears down the device's primary context) it is stale, so do not
 *     call this entry point on a device after resetting it.
 *   - The array is shared by every call and keeps the last call's contents:
 *     two calls that can overlap on the GPU (different streams, or different
 *     host threads without ordering) race on it.  Calls on one stream are
 *     ordered and safe.  Nothing in it needs to start zeroed: the kernels write
 *     each byte they later read.
 *   - Calls no cudaMalloc / cudaFree or any allocating routine.
 */
int b200mm_mla_decode_noalloc(const b200mm_mla_shape* shape,
                              const void* q, int64_t q_sb,
                              const void* c_kv, int64_t c_sb, int64_t c_st,
                              const void* kz, int64_t z_sb, int64_t z_st,
                              const float* kscale, int64_t s_sb, int64_t s_st,
                              const void* w_uk, const void* w_uv,
                              const float* k_norm_w, const float* rope_inv_freq,
                              float scale, int64_t L,
                              void* out, int64_t o_sb,
                              void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200MM_H_ */
