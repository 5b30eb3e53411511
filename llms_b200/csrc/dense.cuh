// Dense projection kernels (fused QKV, fused gate-up-SiLU, int8 weight-only):
// parameter block and dispatch entry shared by the kernel files.
#pragma once
#include "common.cuh"

namespace b200mm {

// One call of the projection family.  y[m, n] = epilogue(x[m,:] . w[n,:]).
//   gate == false : y = acc0 * s0[n]                 (QKV; s0 == nullptr -> 1)
//   gate == true  : y = silu(acc_g * sg[n]) * acc_u * su[n]
struct DenseArgs {
  const void* x; int64_t ldx;       // [M, K] activation dtype
  const void* w0; int64_t ldw0;     // [N, K] (gate or stacked qkv)
  const void* w1; int64_t ldw1;     // [N, K] up weights (gate mode only)
  const float* s0; const float* s1; // per-row scales (int8 weights only)
  void* y; int64_t ldy;             // [M, N] activation dtype
  int M, N, K;
  int dtype;                        // B200MM_F32 / F16 / BF16 (x, y, dense w)
  bool w8;                          // weights are int8
  bool gate;                        // gate-up-SiLU epilogue
  const b200mm_peer_out* peer;      // non-null: store into every rank's gathered buffer (GEMV only)
  cudaStream_t stream;
};

int dense_dispatch(const DenseArgs& a);

// Kernel families (each returns B200MM_OK, or a status if it declines / fails).
// `*_supported` answers whether the family can serve the call, with no launch.
bool gemv_supported(const DenseArgs& a);
int gemv_launch(const DenseArgs& a);
int tiled_launch(const DenseArgs& a);
bool mmv_supported(const DenseArgs& a);
int mmv_launch(const DenseArgs& a);
bool swap_supported(const DenseArgs& a);
int swap_launch(const DenseArgs& a);
bool tc_supported(const DenseArgs& a);
int tc_launch(const DenseArgs& a);

// Decode-step glue (glue.cu); shapes validated by the caller.
int glue_rmsnorm(const void* x, int64_t ldx, const void* r, int64_t ldr, void* h, int64_t ldh, const void* w, void* y,
                 int64_t ldy, int M, int N, float eps, int dtype, cudaStream_t st);
int glue_qk_norm_rope(const void* qkv, int64_t ldq, int B, int H, int KV, int D, const void* qw, const void* kw,
                      const void* cos_t, const void* sin_t, int64_t pos, const int64_t* pos_dev, void* q_out,
                      int64_t q_sb, int64_t q_sh, void* kc, int64_t k_sb, int64_t k_sh, int64_t k_st, void* vc,
                      int64_t v_sb, int64_t v_sh, int64_t v_st, float eps, int dtype, cudaStream_t st);

// GQA single-query decode attention (gqa.cu); shapes validated by the caller.
size_t gqa_workspace_bytes(int B, int H, int KV, int D, int64_t L);
int gqa_decode(const void* q, int64_t q_sb, int64_t q_sh, const void* k, int64_t k_sb, int64_t k_sh, int64_t k_st,
               const void* v, int64_t v_sb, int64_t v_sh, int64_t v_st, void* out, int64_t o_sb, int64_t o_sh,
               int B, int H, int KV, int D, int64_t L, float scale, int dtype, void* ws, size_t ws_bytes,
               cudaStream_t stream);

}  // namespace b200mm
