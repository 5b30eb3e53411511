// MLA latent-KV decode: argument blocks, workspace layout and kernel entry
// points shared between the generic and the production-shape kernels.
#pragma once
#include "tma.cuh"

namespace b200mm {

struct MlaAppendArgs {
  b200mm_mla_shape s;
  const void* c_kv; int64_t c_sb, c_st;
  const void* kr; int64_t r_sb, r_st;     // k_rope_pre
  const void* w_uk;
  const float* k_norm_w; const float* inv_freq;
  float* kscale; int64_t s_sb, s_st;
  void* kz; int64_t z_sb, z_st;
  int64_t t0, t1;
  cudaStream_t stream;
};

struct MlaDecodeArgs {
  b200mm_mla_shape s;
  const void* q; int64_t q_sb;
  const void* c_kv; int64_t c_sb, c_st;
  const void* kz; int64_t z_sb, z_st;     // RoPE'd rope-half side-band
  const float* kscale; int64_t s_sb, s_st;
  const void* w_uk; const void* w_uv;
  const float* k_norm_w; const float* inv_freq;
  float scale; int64_t L;
  void* out; int64_t o_sb;
  void* ws; size_t ws_bytes;
  cudaStream_t stream;
  int64_t qpos;             // position of the query token (L - 1 unless the tokens are a slice of the context)
  float* av_out;            // partial decode: the merged latent of the range [B, H, R] (normalised over it) ...
  float* ml_out;            // ... and its (max score, sum of exp) per (row, head) [B, H, 2]; no W_uv step
};

// Work plan shared by the split kernels and the combine kernel.
// The flattened (batch row, 64-token tile) sequence of T = B * ntiles units
// is cut into G contiguous ranges, range i = [floor(i*T/G), floor((i+1)*T/G)),
// one per CTA of the split kernel.  A CTA writes one partial per batch row
// its range touches, into slot (i + b); batch row b's partials are the slots
// i + b of every range i that overlaps it (so at most G + B slots exist).
//
// Workspace (every region 256-byte aligned):
//   qt   fp32 [B, H, R]        absorbed no-RoPE query  W_uk^T (w_k[:DN] * q[:DN])
//   qr   fp32 [B, H, DR]       RoPE'd query rope half at position L-1
//   pacc fp32 [G+B, H, R]      per-partial sum_t p_t c_t (p relative to the partial max)
//   pml  fp32 [G+B, H, 2]      per-partial (max score, sum p)
//   av   fp32 [B, H, R]        merged sum_t softmax_t c_t (input of the W_uv step)
//   err  int32[4]              error flag of bounded waits (0 = ok)
constexpr int kMlaUnit = 64;  // tokens per work unit

struct MlaWorkspace {
  int G;                  // split CTAs (work ranges)
  int64_t ntiles;         // 64-token units per batch row
  int64_t T;              // B * ntiles
  int rchunks;            // latent chunks per (row, head) in the merge kernel
  int rw;                 // columns per chunk
  size_t off_qt, off_qr, off_pacc, off_pml, off_av, off_err, total;
};

__host__ __device__ inline int64_t mla_range_begin(const MlaWorkspace& w, int i) {
  return (int64_t)i * w.T / w.G;
}

int mla_validate_shape(const b200mm_mla_shape& s);
#ifdef MLA_TC_TRACE
// Development trace (debug builds only): per MLA kernel k (0 absorb, 1 split,
// 2 merge, 3 combine) the earliest start (stored inverted, so one atomicMax
// keeps the minimum) and the latest end, written past the end of the planned
// workspace after the split kernel's own trace.
#define MLA_SPAN(k, end_)                                                                               \
  do {                                                                                                  \
    if (threadIdx.x == 0) {                                                                             \
      unsigned long long* sp_ = reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(a.ws) + \
                                                                      w.total) + (size_t)w.G * 8 * 16; \
      const unsigned long long t_ = global_ns();                                                        \
      atomicMax(&sp_[2 * (k) + (end_)], (end_) ? t_ : ~t_);                                              \
    }                                                                                                   \
  } while (0)
#else
#define MLA_SPAN(k, end_) \
  do {                    \
  } while (0)
#endif

MlaWorkspace mla_plan(const b200mm_mla_shape& s, int64_t L, bool fast);
size_t mla_workspace_bytes(const b200mm_mla_shape& s, int64_t L);
int mla_append_launch(const MlaAppendArgs& a);

// side-band fill on the tensor cores (R=256, D=128, DR=32, KV=8, 16-bit), for
// ranges of at least kMlaFillTcMinTokens tokens per batch row
constexpr int64_t kMlaFillTcMinTokens = 64;
bool mla_fill_tc_supported(const MlaAppendArgs& a);
int mla_fill_tc_launch(const MlaAppendArgs& a);
int mla_decode_launch(const MlaDecodeArgs& a);
// merge per-range partials (part r's av [B][H][R] at av_parts + r * av_stride,
// its ml [B][H][2] at ml_parts + r * ml_stride) into the
// workspace's av, then the W_uv step into a.out
int mla_combine_partials_launch(const MlaDecodeArgs& a, const float* av_parts, int64_t av_stride,
                                const float* ml_parts, int64_t ml_stride, int nparts);

// production-shape split kernel (R=256, D=128, DR=32, H=32, KV=8, 16-bit dtype)
struct MlaMaps {
  CUtensorMap c, kz, ks;  // TMA maps of c_kv, the RoPE'd-key side-band and the k-RMS side-band (token extent = L)
};
bool mla_fast_supported(const MlaDecodeArgs& a);
bool mla_fast_maps(const MlaDecodeArgs& a, MlaMaps* maps);  // false if the driver rejects a map
int mla_fast_ctas();                   // G for the production-shape kernel
int mla_tc_split_launch(const MlaDecodeArgs& a, const MlaWorkspace& w, const MlaMaps& maps);

}  // namespace b200mm
