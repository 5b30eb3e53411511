// MLA latent-KV decode: argument blocks, workspace layout and kernel entry
// points shared between the generic and the production-shape kernels.
#pragma once
#include "common.cuh"

namespace b200mm {

struct MlaScalesArgs {
  b200mm_mla_shape s;
  const void* c_kv; int64_t c_sb, c_st;
  const void* kr; int64_t r_sb, r_st;
  const void* w_uk;
  float* kscale; int64_t s_sb, s_st;
  int64_t t0, t1;
  cudaStream_t stream;
};

struct MlaDecodeArgs {
  b200mm_mla_shape s;
  const void* q; int64_t q_sb;
  const void* c_kv; int64_t c_sb, c_st;
  const void* kr; int64_t r_sb, r_st;
  const float* kscale; int64_t s_sb, s_st;
  const void* w_uk; const void* w_uv;
  const float* k_norm_w; const float* inv_freq;
  float scale; int64_t L;
  void* out; int64_t o_sb;
  void* ws; size_t ws_bytes;
  cudaStream_t stream;
};

// Workspace (fp32, every region 256-byte aligned):
//   qt   [B, H, R]        absorbed no-RoPE query  W_uk^T (w_k[:DN] * q[:DN])
//   qr   [B, H, DR]       RoPE'd query rope half at position L-1
//   pacc [B, S, H, R]     per-split sum_t p_t c_t (p relative to the split max)
//   pml  [B, S, H, 2]     per-split (max score, sum p)
struct MlaWorkspace {
  int S;                  // context splits per batch row
  int64_t chunk;          // tokens per split (the last split may be shorter)
  size_t off_qt, off_qr, off_pacc, off_pml, total;
};

int mla_validate_shape(const b200mm_mla_shape& s);
MlaWorkspace mla_plan(const b200mm_mla_shape& s, int64_t L);
size_t mla_workspace_bytes(const b200mm_mla_shape& s, int64_t L);
int mla_scales_launch(const MlaScalesArgs& a);
int mla_decode_launch(const MlaDecodeArgs& a);

// production-shape split kernel (R=256, D=128, DR=32, H=32, KV=8, 16-bit dtype)
bool mla_fast_supported(const MlaDecodeArgs& a);
int mla_fast_split_launch(const MlaDecodeArgs& a, const MlaWorkspace& w);

}  // namespace b200mm
