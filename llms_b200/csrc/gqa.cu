// GQA decode attention (one query token per sequence) over the engine's KV
// cache: out[b, h] = softmax(q[b, h] . K[b, h / g]^T * scale) V[b, h / g],
// g = H / KV query heads per KV head.  This is the computation behind the
// engine's swappable single-query attention op (`decode_attn_op`, fed the
// pre-expansion K/V of `kv_cache.k[layer][:B, :, :L, :]`).
//
// The step is an HBM stream of the cache (2 * L * D * 2 bytes per sequence and
// KV head; every query head of the group reads the same K/V rows), so the
// production kernel is built around keeping ~190 KB of it in flight per SM:
//   * split kernel, persistent, one CTA per SM.  The flattened sequence of
//     64-token tiles over (row, KV head, context) is cut into one contiguous
//     range per CTA (the plan below); a range may span several (row, KV head)
//     pairs and a pair several ranges;
//   * warp 4 is the producer: per tile one TMA instruction for K and one for
//     V (3-D maps viewing the cache rows as [D / 64][rows][64], 128-byte
//     swizzle), into a 6-stage ring of 32 KB stages (three per group);
//   * warps 0-7 form two groups that take alternate tiles (two tiles in
//     compute at once); each warp of a group owns 16 tokens of the tile.  Scores S^T = Q K^T come
//     from mma.sync m16n8k16 with the group's query heads as the M rows
//     (zero rows past g) and ldmatrix fragments of the swizzled K tile; an
//     online softmax in log2 units runs on the accumulators, which are then
//     reused in registers as the A operand of O += P V (V fragments through
//     ldmatrix.trans).  Tokens past the context length are masked, and their
//     V rows zeroed, so whatever the cache holds there cannot leak;
//   * each warp writes one partial (running max, sum, O rows) per pair its
//     range touches, an empty one if its group got no tile of the pair; a
//     merge kernel over (head, row) combines them.
// Other shapes (fp32, D not 64 / 128, groups above 16, strided token rows)
// run a generic kernel: one CTA per (row, head), scores staged in the
// workspace, two reductions, then O.
#include "dense.cuh"
#include "tma.cuh"

#include <type_traits>

namespace b200mm {

namespace {

constexpr int kTile = 64;        // tokens per tile
constexpr int kStages = 6;
constexpr int kGroups = 2;       // consumer groups, taking alternate tiles
constexpr int kConsumers = 4 * kGroups;  // warps 0-7: group w / 4, 16 tokens (w % 4) of its tiles
// Every stage must serve one group only (tile t lands in stage t % kStages and
// belongs to group t % kGroups).  Otherwise a group running ahead can wait on
// a stage's full barrier two phases on, which a parity wait cannot tell from
// the phase before, and consume a tile that is still in flight.
static_assert(kStages % kGroups == 0, "ring stages must be a multiple of the consumer groups");
constexpr int kGqaThreads = 32 * (kConsumers + 1);
constexpr float kLog2e = 1.4426950408889634f;

struct GqaArgs {
  const void* q; int64_t q_sb, q_sh;                 // [B, H, D]
  const void* k; int64_t k_sb, k_sh, k_st;           // [B, KV, L, D]
  const void* v; int64_t v_sb, v_sh, v_st;
  void* out; int64_t o_sb, o_sh;                     // [B, H, D]
  int B, H, KV, D;
  int64_t L;
  float scale;
  int dtype;
  void* ws; size_t ws_bytes;
  cudaStream_t stream;
};

// Plan of the split kernel: P = B * KV pairs, ntiles tiles per pair,
// T = P * ntiles tiles in all, range i = [floor(i T / G), floor((i+1) T / G)).
// Range i writes its partials for pair p into slot i + p (distinct for every
// (i, p) that meet, as ranges are contiguous); each slot holds one partial per
// consumer warp.  Workspace: int32 [2] error flag and merge counter at byte 0
// (the same place for every shape, zero between calls), then pacc fp32
// [G + P][8][g][D] and pml fp32 [G + P][8][g][2] (max in log2 units, sum).
struct GqaPlan {
  int G, P, g;
  int64_t ntiles, T;
  size_t off_pacc, off_pml, total;
};

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
constexpr size_t kFlagBytes = 256;  // error flag + merge counter, then the data

GqaPlan gqa_plan(int B, int H, int KV, int D, int64_t L, int sms) {
  GqaPlan w{};
  w.P = B * KV;
  w.g = H / KV;
  w.ntiles = (L + kTile - 1) / kTile;
  w.T = (int64_t)w.P * w.ntiles;
  w.G = (int)(sms < w.T ? sms : w.T);
  const size_t slots = (size_t)w.G + w.P;
  w.off_pacc = kFlagBytes;
  w.off_pml = align256(sizeof(float) * slots * kConsumers * w.g * D);
  w.total = align256(w.off_pml + sizeof(float) * slots * kConsumers * w.g * 2);
  return w;
}

// generic path: scores [B, H, L] fp32 after the flag words
size_t generic_ws_bytes(int B, int H, int64_t L) { return kFlagBytes + align256(sizeof(float) * (size_t)B * H * L); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T> struct Mma16816;
template <> struct Mma16816<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Mma16816<__half> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// ---------------------------------------------------------------------------
// split kernel (16-bit, D = 64 or 128, g <= 16, token rows contiguous)
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kGqaThreads, 1)
    gqa_split_kernel(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv,
                     const GqaArgs a, const GqaPlan w, int64_t k_prow, int64_t k_brow, int64_t v_prow,
                     int64_t v_brow, int* err) {
  constexpr int HALVES = D / 64;
  constexpr uint32_t TILE_BYTES = kTile * D * 2;  // one of K / V
  constexpr uint32_t STAGE = 2 * TILE_BYTES;
  constexpr int KS = D / 16;                      // k-steps of the scores
  constexpr int NT = D / 8;                       // n-tiles of O
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStages * STAGE);
  uint64_t* empty = full + kStages;
  volatile int* failed = reinterpret_cast<volatile int*>(empty + kStages);
  int* issued = const_cast<int*>(failed) + 1;  // tiles the producer issued

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x;
  const int64_t r0 = (int64_t)i * w.T / w.G, r1 = (int64_t)(i + 1) * w.T / w.G;
  const int n = (int)(r1 - r0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);  // the four warps of the tile's group
    }
    *failed = 0;
    *issued = 0;
    mbar_init_fence();
    prefetch_map(&mk);
    prefetch_map(&mv);
  }
  __syncthreads();

  // the cache rows of tile k: pair p = k / ntiles (row b = p / KV, head p % KV)
  auto tile_row = [&](int64_t k, int64_t prow, int64_t brow) -> int {  // (k: flattened tile index)
    const int64_t p = k / w.ntiles, j = k - p * w.ntiles;
    return (int)((p / a.KV) * brow + (p % a.KV) * prow + j * kTile);
  };

  if (warp == kConsumers) {
    // ---------------- producer ----------------
    // K and V are written by the kernel that appended this step's token
    pdl_wait();
    if (lane == 0) {
      int t = 0;
      for (; t < n; ++t) {
        const int s = t % kStages;
        if (t >= kStages && !mbar_wait(&empty[s], (uint32_t)(((t - kStages) / kStages) & 1))) {
          *failed = 1;
          break;
        }
        if (*failed) break;
        unsigned char* st = sm + s * STAGE;
        mbar_expect_tx(&full[s], STAGE);
        tma_load_3d(st, &mk, 0, tile_row(r0 + t, k_prow, k_brow), 0, &full[s]);
        tma_load_3d(st + TILE_BYTES, &mv, 0, tile_row(r0 + t, v_prow, v_brow), 0, &full[s]);
      }
      *issued = t;
    }
  } else {
    // ---------------- consumers ----------------
    using M = Mma16816<T>;
    pdl_wait();  // q comes from the previous kernels
    const int hq = lane >> 2;           // this lane's head rows: hq and hq + 8
    const int tq = 2 * (lane & 3);      // this lane's token columns within an n-tile: tq, tq + 1
    const float sl2 = a.scale * kLog2e;
    uint32_t qa[KS][4];
    float o[NT][4];
    float mrow[2], lrow[2];
    int64_t cur = -1;                   // pair of the running partial
    bool ok = true;

    auto load_q = [&](int64_t p) {
      const int b = (int)(p / a.KV), kvh = (int)(p % a.KV);
      const T* qb = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)kvh * w.g * a.q_sh;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int h = hq + 8 * (r & 1), d = 16 * ks + tq + 8 * (r >> 1);
          uint32_t v = 0;
          if (h < w.g) v = *reinterpret_cast<const uint32_t*>(qb + (int64_t)h * a.q_sh + d);
          qa[ks][r] = v;
        }
      }
    };
    auto reset = [&]() {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
      mrow[0] = mrow[1] = -INFINITY;
      lrow[0] = lrow[1] = 0.f;
    };
    auto flush = [&](int64_t p) {  // this warp's partial for pair p -> slot (i + p), warp
      float l0 = lrow[0], l1 = lrow[1];
      l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
      l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
      const int64_t slot = ((int64_t)i + p) * kConsumers + warp;
      float* ws = static_cast<float*>(a.ws);
      float* pacc = ws + w.off_pacc / 4 + slot * w.g * D;
      float* pml = ws + w.off_pml / 4 + slot * w.g * 2;
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int h = hq + 8 * hr;
        if (h < w.g) {
#pragma unroll
          for (int j = 0; j < NT; ++j)
            *reinterpret_cast<float2*>(pacc + (int64_t)h * D + 8 * j + tq) = make_float2(o[j][2 * hr], o[j][2 * hr + 1]);
          if ((lane & 3) == 0) {
            pml[2 * h] = mrow[hr];
            pml[2 * h + 1] = hr ? l1 : l0;
          }
        }
      }
    };

    const int grp = warp >> 2;
    for (int t = 0; ok && t < n; ++t) {
      const int64_t k = r0 + t;
      const int64_t p = k / w.ntiles;
      if (p != cur) {  // every warp sees every pair of the range, so each writes its partial
        if (cur >= 0) flush(cur);
        cur = p;
        load_q(p);
        reset();
      }
      if ((t % kGroups) != grp) continue;
      const int s = t % kStages;
      if (!mbar_wait(&full[s], (uint32_t)((t / kStages) & 1)) || *failed) {
        ok = false;
        break;
      }
      const int64_t j = k - p * w.ntiles;
      const int nv = (int)(a.L - j * kTile < kTile ? a.L - j * kTile : kTile);  // valid tokens of the tile
      const uint32_t kbase = smem_u32(sm + s * STAGE), vbase = kbase + TILE_BYTES;
      const int t0 = 16 * (warp & 3);  // this warp's first token row of the tile

      const bool zeroed = t0 + 16 > nv;
      if (zeroed) {
        // zero this warp's V rows past the context (the cache may hold anything there)
        unsigned char* vrow = sm + s * STAGE + TILE_BYTES;
        for (int e = lane; e < 16 * HALVES * 8; e += 32) {
          const int rr = t0 + e / (HALVES * 8), hh = (e / 8) % HALVES, c = e % 8;
          if (rr >= nv) *reinterpret_cast<uint4*>(vrow + hh * kTile * 128 + rr * 128 + c * 16) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }

      // scores: S^T[h, t0 + 0..15] in two n-tiles of 8 tokens
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        // matrices: (rows t0..+7, chunk c), (t0..+7, c+1), (t0+8.., c), (t0+8.., c+1)
        const int row = t0 + (lane & 7) + ((lane >> 4) << 3);
        const int col = 16 * ks + 8 * ((lane >> 3) & 1);
        const int hh = col >> 6, c = (col >> 3) & 7;
        const uint32_t addr = kbase + hh * kTile * 128 + row * 128 + ((c ^ (row & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        M::run(sc[0], qa[ks], b0, b1);
        M::run(sc[1], qa[ks], b2, b3);
      }
      // online softmax per head row (log2 units); masked tokens -> -inf
      float mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = t0 + 8 * nt + tq + (e & 1);
          const float v = tok < nv ? sc[nt][e] * sl2 : -INFINITY;
          sc[nt][e] = v;
          mt[e >> 1] = fmaxf(mt[e >> 1], v);
        }
      float fac[2];
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        mt[hr] = fmaxf(mt[hr], __shfl_xor_sync(0xffffffffu, mt[hr], 1));
        mt[hr] = fmaxf(mt[hr], __shfl_xor_sync(0xffffffffu, mt[hr], 2));
        const float mn = fmaxf(mrow[hr], mt[hr]);
        fac[hr] = mn == -INFINITY ? 1.f : exp2f(mrow[hr] - mn);
        mrow[hr] = mn;
        lrow[hr] *= fac[hr];
      }
      uint32_t pa[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        float pv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int hr = e >> 1;
          pv[e] = mrow[hr] == -INFINITY ? 0.f : exp2f(sc[nt][e] - mrow[hr]);
          lrow[hr] += pv[e];
        }
        // A fragment of P (rows = heads, k = the 16 tokens): n-tile 0 -> a0/a1, n-tile 1 -> a2/a3
        pa[2 * nt] = M::pack(pv[0], pv[1]);
        pa[2 * nt + 1] = M::pack(pv[2], pv[3]);
      }
#pragma unroll
      for (int jn = 0; jn < NT; ++jn) {
        o[jn][0] *= fac[0]; o[jn][1] *= fac[0];
        o[jn][2] *= fac[1]; o[jn][3] *= fac[1];
      }
      // O[h, d] += P[h, t] V[t, d]; V fragments by ldmatrix.trans, two n-tiles per load
#pragma unroll
      for (int jp = 0; jp < NT / 2; ++jp) {
        // matrices: (rows t0..+7, chunk c), (t0+8..+15, c), (t0..+7, c+1), (t0+8.., c+1)
        const int row = t0 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int col = 16 * jp + 8 * (lane >> 4);
        const int hh = col >> 6, c = (col >> 3) & 7;
        const uint32_t addr = vbase + hh * kTile * 128 + row * 128 + ((c ^ (row & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(addr, b0, b1, b2, b3);
        M::run(o[2 * jp], pa, b0, b1);
        M::run(o[2 * jp + 1], pa, b2, b3);
      }
      if (zeroed) fence_proxy_async();  // generic writes before the next TMA write of this stage
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (ok && cur >= 0) flush(cur);
    if (!ok) *failed = 1;
  }
  pdl_trigger();
  __syncthreads();
  if (threadIdx.x == 0 && *failed) {
    atomicExch(err, 1);
    // copies issued but never consumed still target this CTA's shared memory:
    // wait for the last issued tile of every stage
    const int iss = *issued;
    for (int t = iss > kStages ? iss - kStages : 0; t < iss; ++t)
      mbar_wait(&full[t % kStages], (uint32_t)((t / kStages) & 1));
  }
}

// ---------------------------------------------------------------------------
// merge: out[b, h] = sum_k 2^(m_k - M) O_k / sum_k 2^(m_k - M) l_k
// grid (H, B), block 256: warp 0 weighs the partials, then warp w sums
// partials w, w + 8, ... with lane = 4 output dims (independent float4 loads,
// so a pair spread over many ranges does not become one long load chain),
// and a shared-memory sum over the warps finishes.
// ---------------------------------------------------------------------------
constexpr int kMergeThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kMergeThreads) gqa_merge_kernel(const GqaArgs a, const GqaPlan w, int* err) {
  extern __shared__ float msm[];  // [8][D] warp sums, then [partials] weights
  __shared__ float s_inv;
  const int D = a.D;
  float* red = msm;
  float* wgt = msm + (kMergeThreads / 32) * D;
  const int h = blockIdx.x, b = blockIdx.y;
  const int kvh = h / w.g, hl = h % w.g;
  const int64_t p = (int64_t)b * a.KV + kvh;
  const int64_t lo = p * w.ntiles, hi = lo + w.ntiles;
  const int i0 = (int)(((lo + 1) * w.G - 1) / w.T);  // ranges overlapping [lo, hi)
  const int i1 = (int)((hi * w.G - 1) / w.T);
  const int np = (i1 - i0 + 1) * kConsumers;
  const float* ws = static_cast<const float*>(a.ws);
  const float* pml = ws + w.off_pml / 4;
  const float* pacc = ws + w.off_pacc / 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  auto slot_of = [&](int k) { return ((int64_t)i0 + k / kConsumers + p) * kConsumers + k % kConsumers; };
  __shared__ float s_red[kMergeThreads / 32];
  // weights of the partials, all threads at once: block max, then 2^(m - max)
  float mx = -INFINITY;
  for (int k = threadIdx.x; k < np; k += kMergeThreads) {
    const float m = pml[(slot_of(k) * w.g + hl) * 2];
    wgt[k] = m;
    mx = fmaxf(mx, m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  mx = s_red[0];
#pragma unroll
  for (int k = 1; k < kMergeThreads / 32; ++k) mx = fmaxf(mx, s_red[k]);
  float l = 0.f;
  for (int k = threadIdx.x; k < np; k += kMergeThreads) {
    const float m = wgt[k];
    const float e = m == -INFINITY ? 0.f : exp2f(m - mx);
    wgt[k] = e;
    l += e * pml[(slot_of(k) * w.g + hl) * 2 + 1];
  }
  l = warp_sum(l);
  __syncthreads();  // every warp has read s_red
  if (lane == 0) s_red[warp] = l;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kMergeThreads / 32; ++k) t += s_red[k];
    s_inv = 1.f / t;
  }
  __syncthreads();
  const int d4 = 4 * lane;
  if (d4 < D) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int k = warp; k < np; k += kMergeThreads / 32) {
      const float e = wgt[k];
      const float4 v = *reinterpret_cast<const float4*>(pacc + (slot_of(k) * w.g + hl) * D + d4);
      acc.x = fmaf(e, v.x, acc.x); acc.y = fmaf(e, v.y, acc.y);
      acc.z = fmaf(e, v.z, acc.z); acc.w = fmaf(e, v.w, acc.w);
    }
    *reinterpret_cast<float4*>(red + warp * D + d4) = acc;
  }
  __syncthreads();
  const bool bad = *reinterpret_cast<volatile int*>(err) != 0;
  for (int d = threadIdx.x; d < D; d += kMergeThreads) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kMergeThreads / 32; ++k) acc += red[k * D + d];
    float v = acc * s_inv;
    if (bad) v = __int_as_float(0x7fc00000);
    static_cast<T*>(a.out)[(int64_t)b * a.o_sb + (int64_t)h * a.o_sh + d] = from_f<T>(v);
  }
  // the last CTA to finish clears the error flag and the counter for the next
  // call (every CTA read the flag above, before counting itself)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned n = gridDim.x * gridDim.y;
    if (atomicAdd(reinterpret_cast<unsigned*>(err) + 1, 1u) == n - 1) {
      err[0] = 0;
      err[1] = 0;
    }
  }
  pdl_trigger();
}

// ---------------------------------------------------------------------------
// generic: one CTA per (head, row); scores to the workspace
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) gqa_generic_kernel(const GqaArgs a) {
  __shared__ float red[32];
  __shared__ float s_m, s_inv;
  const int h = blockIdx.x, b = blockIdx.y;
  const int kvh = h / (a.H / a.KV);
  const T* q = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)h * a.q_sh;
  const T* kb = static_cast<const T*>(a.k) + (int64_t)b * a.k_sb + (int64_t)kvh * a.k_sh;
  const T* vb = static_cast<const T*>(a.v) + (int64_t)b * a.v_sb + (int64_t)kvh * a.v_sh;
  float* sc = reinterpret_cast<float*>(static_cast<unsigned char*>(a.ws) + kFlagBytes) + ((int64_t)b * a.H + h) * a.L;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  pdl_wait();
  // scores, one warp per token
  float mx = -INFINITY;
  for (int64_t t = warp; t < a.L; t += nw) {
    const T* kr = kb + t * a.k_st;
    float s = 0.f;
    for (int d = lane; d < a.D; d += 32) s = fmaf(to_f<T>(q[d]), to_f<T>(kr[d]), s);
    s = warp_sum(s) * a.scale;
    if (lane == 0) sc[t] = s;
    mx = fmaxf(mx, s);
  }
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int k = 0; k < nw; ++k) m = fmaxf(m, red[k]);
    s_m = m;
  }
  __syncthreads();
  float l = 0.f;
  for (int64_t t = threadIdx.x; t < a.L; t += blockDim.x) {
    const float e = expf(sc[t] - s_m);
    sc[t] = e;
    l += e;
  }
  l = warp_sum(l);
  __syncthreads();
  if (lane == 0) red[warp] = l;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int k = 0; k < nw; ++k) s += red[k];
    s_inv = 1.f / s;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
    float acc = 0.f;
    for (int64_t t = 0; t < a.L; ++t) acc = fmaf(sc[t], to_f<T>(vb[t * a.v_st + d]), acc);
    static_cast<T*>(a.out)[(int64_t)b * a.o_sb + (int64_t)h * a.o_sh + d] = from_f<T>(acc * s_inv);
  }
  pdl_trigger();
}

bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

bool fast_ok(const GqaArgs& a) {
  if (g_force_generic.load(std::memory_order_relaxed)) return false;
  if (a.dtype != B200MM_BF16 && a.dtype != B200MM_F16) return false;
  if (a.D != 64 && a.D != 128) return false;
  if (a.H / a.KV > 16) return false;
  if (a.k_st != a.D || a.v_st != a.D) return false;
  if (a.k_sb % a.D || a.k_sh % a.D || a.v_sb % a.D || a.v_sh % a.D) return false;
  if (!al16(a.k) || !al16(a.v) || !al16(a.q)) return false;
  if ((a.q_sh * 2) % 4 || (a.q_sb * 2) % 4) return false;  // 4-byte query pair loads
  // the flattened cache row of every tile start must fit the map's int32 coordinate
  const int64_t rows = (int64_t)(a.B - 1) * (a.k_sb / a.D) + (int64_t)(a.KV - 1) * (a.k_sh / a.D) + a.L;
  const int64_t vrows = (int64_t)(a.B - 1) * (a.v_sb / a.D) + (int64_t)(a.KV - 1) * (a.v_sh / a.D) + a.L;
  return rows < (int64_t(1) << 31) && vrows < (int64_t(1) << 31);
}

template <typename T, int D>
int launch_fast(const GqaArgs& a) {
  const int dev = current_device();
  const GqaPlan w = gqa_plan(a.B, a.H, a.KV, a.D, a.L, num_sms(dev));
  int* err = static_cast<int*>(a.ws);  // [0] error flag, [1] merge counter
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int64_t krows = (int64_t)(a.B - 1) * (a.k_sb / D) + (int64_t)(a.KV - 1) * (a.k_sh / D) + a.L;
  const int64_t vrows = (int64_t)(a.B - 1) * (a.v_sb / D) + (int64_t)(a.KV - 1) * (a.v_sh / D) + a.L;
  CUtensorMap mk, mv;
  if (!make_map_3d(&mk, dt, a.k, 64, (uint64_t)krows, D / 64, (uint64_t)D * 2, 128, 64, kTile, D / 64,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_3d(&mv, dt, a.v, 64, (uint64_t)vrows, D / 64, (uint64_t)D * 2, 128, 64, kTile, D / 64,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return B200MM_ERR_ALIGN;
  constexpr size_t smem = (size_t)kStages * 2 * kTile * D * 2 + 1024 + 256;
  auto split = gqa_split_kernel<T, D>;
  static bool configured[64] = {false};
  if (dev < 0 || dev >= 64) return B200MM_ERR_DEVICE;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(split, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return B200MM_ERR_LAUNCH;
    configured[dev] = true;
  }
  cudaError_t e = launch_pdl(split, dim3(w.G), dim3(kGqaThreads), smem, a.stream, mk, mv, a, w, a.k_sh / D,
                             a.k_sb / D, a.v_sh / D, a.v_sb / D, err);
  if (e != cudaSuccess) return B200MM_ERR_LAUNCH;
  const int maxp = (int)((w.ntiles * w.G + w.T - 1) / w.T + 2) * kConsumers;
  e = launch_pdl(gqa_merge_kernel<T>, dim3(a.H, a.B), dim3(kMergeThreads),
                 sizeof(float) * ((kMergeThreads / 32) * D + maxp), a.stream, a, w, err);
  return e == cudaSuccess ? B200MM_OK : B200MM_ERR_LAUNCH;
}

template <typename T>
int launch_generic(const GqaArgs& a) {
  cudaError_t e = launch_pdl(gqa_generic_kernel<T>, dim3(a.H, a.B), dim3(256), 0, a.stream, a);
  return e == cudaSuccess ? B200MM_OK : B200MM_ERR_LAUNCH;
}

}  // namespace

size_t gqa_workspace_bytes(int B, int H, int KV, int D, int64_t L) {
  const GqaPlan w = gqa_plan(B, H, KV, D, L, num_sms(current_device()));
  const size_t fast = w.total;
  const size_t gen = generic_ws_bytes(B, H, L);
  return fast > gen ? fast : gen;
}

int gqa_decode(const void* q, int64_t q_sb, int64_t q_sh, const void* k, int64_t k_sb, int64_t k_sh, int64_t k_st,
               const void* v, int64_t v_sb, int64_t v_sh, int64_t v_st, void* out, int64_t o_sb, int64_t o_sh,
               int B, int H, int KV, int D, int64_t L, float scale, int dtype, void* ws, size_t ws_bytes,
               cudaStream_t stream) {
  GqaArgs a{q, q_sb, q_sh, k, k_sb, k_sh, k_st, v, v_sb, v_sh, v_st, out, o_sb, o_sh,
            B, H, KV, D, L, scale, dtype, ws, ws_bytes, stream};
  if (ws_bytes < gqa_workspace_bytes(B, H, KV, D, L)) return B200MM_ERR_WORKSPACE;
  if (fast_ok(a)) {
    if (dtype == B200MM_BF16)
      return D == 128 ? launch_fast<__nv_bfloat16, 128>(a) : launch_fast<__nv_bfloat16, 64>(a);
    return D == 128 ? launch_fast<__half, 128>(a) : launch_fast<__half, 64>(a);
  }
  if (dtype == B200MM_BF16) return launch_generic<__nv_bfloat16>(a);
  if (dtype == B200MM_F16) return launch_generic<__half>(a);
  return launch_generic<float>(a);
}

}  // namespace b200mm
