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

// ---------------------------------------------------------------------------
// Peer output (the b200mm_*_peer entry points): a projection's epilogue
// stores column n of this rank's shard into every rank's gathered buffer, at
// the column an all-gather would give it, and the launch ends with one
// completion count per peer and a bounded wait for the peers' counts.
// ---------------------------------------------------------------------------
struct PeerEpi {
  int world, rank, nparts;  // world == 0: no peer output
  int64_t ld;               // gathered row stride (elements)
  int64_t pw[3], pdoff[3];  // part widths; part j's rank-0 column in the gathered row
  void* pdst[8];
  unsigned* pflags[8];
  unsigned* ticket;
  unsigned* seen;
  int* err;
};

inline void peer_epi_from(const b200mm_peer_out& po, PeerEpi& e) {
  e.world = po.world;
  e.rank = po.rank;
  e.nparts = po.nparts;
  e.ld = po.ld_dst;
  int64_t off = 0;
  for (int j = 0; j < po.nparts; ++j) {
    e.pw[j] = po.part_widths[j];
    e.pdoff[j] = off;
    off += po.part_widths[j] * po.world;
  }
  for (int r = 0; r < po.world; ++r) {
    e.pdst[r] = po.dst[r];
    e.pflags[r] = static_cast<unsigned*>(po.flags[r]);
  }
  e.ticket = static_cast<unsigned*>(po.ticket);
  e.seen = static_cast<unsigned*>(po.seen);
  e.err = static_cast<int*>(po.err);
}

constexpr unsigned long long kPeerWaitNs = 5ull * 1000 * 1000 * 1000;  // 5 s

__device__ __forceinline__ int64_t peer_col(const PeerEpi& e, int n) {
  int64_t c = n;
  int j = 0;
  while (j + 1 < e.nparts && c >= e.pw[j]) c -= e.pw[j++];
  return e.pdoff[j] + (int64_t)e.rank * e.pw[j] + c;
}

// Row `row`, shard column n, value v -> every rank's gathered buffer.
template <typename TX>
__device__ __forceinline__ void peer_store(const PeerEpi& e, int64_t row, int n, TX v) {
  const int64_t d = row * e.ld + peer_col(e, n);
  for (int r = 0; r < e.world; ++r) static_cast<TX*>(e.pdst[r])[d] = v;
}

// End of a peer-output launch (every thread of every CTA calls it): each CTA
// takes a ticket with a release (after a barrier, so it covers the CTA's
// stores); the launch's last CTA, whose ticket acquires all of them, counts
// the launch done on every peer with a system-scope release add (cumulative:
// it carries the other CTAs' stores too; one remote add per peer, not one per
// CTA) and then waits (bounded) until every peer's launch has counted itself
// done here.  A full system fence per CTA instead cost ~8 us per launch.
__device__ __forceinline__ void peer_finish(const PeerEpi& e) {
  __syncthreads();  // the CTA's stores are issued
  if (threadIdx.x != 0) return;
  const unsigned ncta = gridDim.x * gridDim.y * gridDim.z;
  unsigned t;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(t) : "l"(e.ticket) : "memory");
  if (t + 1 != ncta) return;
  atomicExch(e.ticket, 0u);  // the next launch on this stream starts after this one ends
  for (int r = 0; r < e.world; ++r)
    if (r != e.rank)
      asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(e.pflags[r] + e.rank) : "memory");
  const unsigned expect = *e.seen + 1u;
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (int r = 0; r < e.world; ++r) {
    if (r == e.rank) continue;
    for (;;) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(e.pflags[e.rank] + r) : "memory");
      if ((int)(v - expect) >= 0) break;
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (now - t0 > kPeerWaitNs) {
        atomicExch(e.err, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  *e.seen = expect;
}

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
