// Mid-M projection kernel on 5th-generation tensor cores, weights as the MMA's
// M operand ("swap-AB"):
//
//   Y^T[f, m] = sum_k W[f, k] X[m, k]          (QKV; int8: times s[f])
//   Y[m, f]   = silu(G[f, m]) * U[f, m]         (gate-up; int8: G, U scaled)
//
// Decode and small-batch calls have few activation rows, so they go on the
// MMA's N side (N = 16..64; int8 weights up to 256 per tile, any M) and the
// weight rows fill the accumulator lanes.
// One CTA owns 128 weight rows (16-bit weights) or 64 (int8) and an N-tile of
// activation rows.  The tensor core takes about 85 ns per small-N instruction
// (measured, N = 16..64, whether one thread or four issue them), so at M = 64
// it, not HBM, set the pace: 128-row tiles move twice the weight bytes per
// instruction, and the K split below restores the CTA count.
//
// The kernel is a weight stream, so its speed is the bytes it keeps in flight:
// at full load HBM answers in about 3 us, and 6 TB/s needs ~190 KB in flight
// per streaming SM.  The producer therefore fetches up to eight K-chunks per
// TMA instruction (3-D tensor maps viewing [rows, K] as [K / 64][rows][64])
// into a ring sized at launch: ~200 KB when every tile has an SM of its own,
// ~100 KB when two CTAs share an SM.  Big stages also mean few
// tcgen05.commit releases, each of which stalls the issuing thread.  K may also be split over a thread-block cluster
// (only when all the tile clusters are resident at once); the ranks reduce
// through distributed shared memory into rank 0, which runs the epilogue.
//
// Warps: 0 TMA producer, 1 TMEM owner + MMA issuer (the K steps rotate over
// up to four accumulator sets: back-to-back small MMAs into one accumulator
// wait on each other), 2-5 int8 -> fp16
// converters (int8 weights: the staged int8 chunks become fp16 in a 2-deep
// operand ring; int8 is exact in fp16, and the activations are converted to
// fp16 for those calls since the MMA takes one type for both operands) and
// the epilogue.  Every mbarrier wait is bounded; a CTA whose wait expires
// stops, drains its copies in flight, and its outputs become NaN.
#include "dense.cuh"
#include "tcgen05.cuh"

#include <cstdlib>
#include <type_traits>

namespace b200mm {

namespace {

constexpr int BK = 64;     // K per chunk (128 bytes of 16-bit elements)
constexpr int kThr = 192;  // warps: 0 TMA, 1 MMA issuer + TMEM owner, 2-5 converters + epilogue
constexpr int kMaxNS = 16;  // ring stages (barrier arrays)
constexpr uint32_t kBudget1 = 200 * 1024, kBudget2 = 100 * 1024;  // ring bytes: one / two CTAs per SM

template <int MN, bool GATE, bool W8>
struct SwapCfg {
  // weight rows per CTA = MMA M: 128 for 16-bit weights (a small-N MMA costs
  // about the same at M = 64 and M = 128, and the tensor core, not HBM, set
  // the pace of the M = 64 tiles); 64 for int8, whose converter hand-off is
  // the limit and whose fp16 operand ring would not fit beside 128-row tiles
  static constexpr int FM = W8 ? 64 : 128;
  static constexpr int NW = GATE ? 2 : 1;
  static constexpr uint32_t W16 = FM * BK * 2;  // 16-bit weight chunk
  static constexpr uint32_t WB = W8 ? FM * BK : W16;  // staged weight chunk
  static constexpr uint32_t XB = MN * BK * 2;   // activation chunk
  static constexpr uint32_t CHUNK = NW * WB + XB;  // staged bytes per K-chunk
  static constexpr uint32_t OPST = W8 ? NW * W16 + XB : 0;  // converted operands of one chunk
  static constexpr int OPS = W8 ? 2 : 0;
  static constexpr int ACC = NW * MN;           // accumulator columns
  static constexpr int CW = ACC >= 32 ? 32 : 16;  // accumulator columns per TMEM load
  static constexpr int SPAN = MN < CW ? MN : CW;  // activation columns per epilogue block
  static constexpr int NB = MN / SPAN;            // epilogue blocks; block j belongs to cluster rank j % cs
  // floats per partial row at an owner rank: its blocks only, gate and up
  __host__ __device__ static constexpr int rpo(int cs) { return (NB + cs - 1) / cs * SPAN * NW + 4; }
  // bytes an owner rank receives from the other cs - 1 ranks
  __host__ __device__ static constexpr uint32_t red_bytes(int cs) {
    return (uint32_t)(cs - 1) * FM * rpo(cs) * 4;
  }
  static constexpr uint32_t EXTRA = 1024 /*align*/ + 512 /*barriers, flags*/;
  static_assert(WB % 1024 == 0 && XB % 1024 == 0 && OPST % 1024 == 0, "chunks must keep the 1024-byte alignment");
};

struct SwapParams {
  const float* s0;
  const float* s1;
  void* y;
  int64_t ldy;
  int M, N, K;
  int nstages;  // K stages in all: ceil(ceil(K / 64) / kc)
  int kc;       // K-chunks per stage (one TMA instruction per operand)
  int map3d;    // 3-D [K / 64][rows][64] maps (else 2-D, kc == 1)
  int ns;       // ring depth
  int cs;       // cluster size (K split)
  int na;       // accumulator sets the K steps rotate over
  uint32_t tmem_cols;
  int debug;    // trace builds only: 1 = no MMAs, 2 = no activation loads
};

#ifdef SWAP_TRACE
// Development trace (debug builds only): per CTA (first 64), %globaltimer at
// the producer's issue and the issuer's start of stages 0-23, plus epilogue
// start / end; read back with b200mm_debug_trace.
__device__ unsigned long long g_swap_trace[64][3][24];
#define STRACE(what, i)                                                       \
  do {                                                                        \
    const unsigned cta_ = blockIdx.x + gridDim.x * blockIdx.y;                \
    if (cta_ < 64 && (i) < 24) g_swap_trace[cta_][(what)][(i)] = global_ns(); \
  } while (0)
#else
#define STRACE(what, i) \
  do {                  \
  } while (0)
#endif

template <int W>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v) {
  if constexpr (W == 32)
    tmem_ld32(taddr, v);
  else
    tmem_ld16(taddr, v);
}

template <typename T, int MN, bool GATE, bool W8>
__global__ void __launch_bounds__(kThr, 2)
    tc_swap_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mw0,
                   const __grid_constant__ CUtensorMap mw1, const SwapParams p) {
  using C = SwapCfg<MN, GATE, W8>;
  using TM = typename std::conditional<W8, __half, T>::type;  // MMA operand type
  constexpr int FM = C::FM;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  const uint32_t STAGE = (uint32_t)p.kc * C::CHUNK;
  const uint32_t RING = (uint32_t)p.ns * STAGE;
  unsigned char* ops = sm + RING;  // converted-operand ring (int8 path)
  uint64_t* full = reinterpret_cast<uint64_t*>(ops + C::OPS * C::OPST);
  uint64_t* empty = full + kMaxNS;
  uint64_t* ofull = empty + kMaxNS;
  uint64_t* oempty = ofull + 2;
  uint64_t* accum = oempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued = const_cast<int*>(failed) + 1;
  int* consumed = issued + 1;
  int* peer_failed = consumed + 1;  // set by another rank of the cluster

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) STRACE(2, 2);
  const int rank = p.cs > 1 ? (int)cluster_rank() : 0;
  const int f0 = (blockIdx.x / p.cs) * FM, m0 = blockIdx.y * MN;
  const int st0 = (int)((int64_t)rank * p.nstages / p.cs), st1 = (int)((int64_t)(rank + 1) * p.nstages / p.cs);
  const int nst = st1 - st0;  // K stages of this CTA
  const int ns = p.ns, kc = p.kc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W8 ? 128 : 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&ofull[s], 128);
      mbar_init(&oempty[s], 1);
    }
    mbar_init(accum, 1);
    *failed = 0;
    *issued = 0;
    *consumed = 0;
    *peer_failed = 0;
    mbar_init_fence();
    prefetch_map(&mx);
    prefetch_map(&mw0);
    if (GATE) prefetch_map(&mw1);
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_trigger();
  pdl_wait();  // X may be the output of the previous kernel
  if (threadIdx.x == 0) STRACE(2, 3);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int i = 0;
      for (; i < nst; ++i) {
        const int s = i % ns;
        if (i >= ns && !mbar_wait(&empty[s], (uint32_t)(((i - ns) / ns) & 1))) {
          *failed = 1;
          break;
        }
        if (*failed) break;
        const int chunk = (st0 + i) * kc;  // first K-chunk of the stage
        unsigned char* st = sm + s * STAGE;
        STRACE(0, i);
        const bool nox = (p.debug & 2) != 0;
        mbar_expect_tx(&full[s], nox ? STAGE - kc * C::XB : STAGE);
        unsigned char* xdst = st + C::NW * kc * C::WB;
        if (p.map3d) {  // one instruction per operand brings kc chunks: [kc][rows][64]
          tma_load_3d(st, &mw0, 0, f0, chunk, &full[s]);
          if (GATE) tma_load_3d(st + kc * C::WB, &mw1, 0, f0, chunk, &full[s]);
          if (!nox) tma_load_3d(xdst, &mx, 0, m0, chunk, &full[s]);
        } else {
          tma_load_2d(st, &mw0, chunk * BK, f0, &full[s]);
          if (GATE) tma_load_2d(st + C::WB, &mw1, chunk * BK, f0, &full[s]);
          tma_load_2d(xdst, &mx, chunk * BK, m0, &full[s]);
        }
      }
      *issued = i;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // Consecutive MMAs into one accumulator wait for each other, which costs
    // small-N instructions several times their issue time; the K steps
    // rotate over `na` accumulator sets instead, summed in the epilogue.
    if (lane == 0) {
      constexpr uint32_t ID = idesc_f16<TM>(FM, MN);
      const int na = p.na;
      int i = 0, mine = 0;
      bool ok = true;
      for (; ok && i < nst; ++i) {
        const int s = i % ns;
        if (!W8) {
          if (!mbar_wait(&full[s], (uint32_t)((i / ns) & 1)) || *failed) {
            ok = false;
            break;
          }
          STRACE(1, i);
          tc_fence_after();
        }
        for (int c = 0; c < kc; ++c) {
          const int g = i * kc + c;  // local chunk index
          uint32_t w0a, w1a, xa;
          if (W8) {
            if (!mbar_wait(&ofull[g & 1], (uint32_t)((g >> 1) & 1)) || *failed) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t base = smem_u32(ops + (g & 1) * C::OPST);
            w0a = base;
            w1a = base + C::W16;
            xa = base + C::NW * C::W16;
          } else {
            const uint32_t base = smem_u32(sm + s * STAGE);
            w0a = base + c * C::W16;
            w1a = base + (kc + c) * C::W16;
            xa = base + C::NW * kc * C::W16 + c * C::XB;
          }
          const uint64_t a0 = sdesc(w0a), a1 = sdesc(w1a), b = sdesc(xa);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            if (p.debug & 1) break;
            const uint32_t acc = tmem + (uint32_t)((kk % na) * C::ACC);
            const uint32_t first = (mine == 0 && kk < na) ? 0u : 1u;
            mma_f16(acc, a0 + 2 * kk, b + 2 * kk, ID, first);
            if (GATE) mma_f16(acc + MN, a1 + 2 * kk, b + 2 * kk, ID, first);
          }
          ++mine;
          if (W8) mma_commit(&oempty[g & 1]);
        }
        if (!ok) break;
        if (!W8) mma_commit(&empty[s]);
      }
      if (!ok) *failed = 1;
      if (!W8) *consumed = i;
      mma_commit(accum);  // fires once every MMA issued above has completed
    }
  } else if (W8 && warp >= 2 && warp <= 5) {
    // ---------------- int8 -> fp16 converters (warps 2-5) ----------------
    const int gt = threadIdx.x - 64;
    int i = 0;
    for (; i < nst; ++i) {
      const int s = i % ns;
      bool ok = mbar_wait(&full[s], (uint32_t)((i / ns) & 1));
      if (gt == 0) STRACE(1, i);
      const unsigned char* st = sm + s * STAGE;
      for (int c = 0; ok && c < kc; ++c) {
        const int g = i * kc + c, o = g & 1;
        if (g >= 2) ok = mbar_wait(&oempty[o], (uint32_t)(((g - 2) >> 1) & 1));
        if (!ok || *failed) break;
        unsigned char* op = ops + o * C::OPST;
        // weights: [64 rows x 64 int8] dense -> [64 rows x 128 B] fp16, swizzled
#pragma unroll
        for (int wsel = 0; wsel < C::NW; ++wsel) {
#pragma unroll
          for (int it = gt; it < FM * 4; it += 128) {
            const int row = it >> 2, c4 = it & 3;
            const uint4 q = *reinterpret_cast<const uint4*>(st + (wsel * kc + c) * C::WB + row * 64 + c4 * 16);
            const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
            uint4 lo, hi;
            lo.x = i8x2_to_h2(w[0], 0); lo.y = i8x2_to_h2(w[0], 1);
            lo.z = i8x2_to_h2(w[1], 0); lo.w = i8x2_to_h2(w[1], 1);
            hi.x = i8x2_to_h2(w[2], 0); hi.y = i8x2_to_h2(w[2], 1);
            hi.z = i8x2_to_h2(w[3], 0); hi.w = i8x2_to_h2(w[3], 1);
            unsigned char* dst = op + wsel * C::W16 + row * 128;
            *reinterpret_cast<uint4*>(dst + (((2 * c4) ^ (row & 7)) << 4)) = lo;
            *reinterpret_cast<uint4*>(dst + (((2 * c4 + 1) ^ (row & 7)) << 4)) = hi;
          }
        }
        // activations: same swizzled positions, converted to fp16
        {
          const unsigned char* xs = st + C::NW * kc * C::WB + c * C::XB;
          unsigned char* xd = op + C::NW * C::W16;
          for (int it = gt; it < MN * 8; it += 128) {
            uint4 v = *reinterpret_cast<const uint4*>(xs + it * 16);
            if (std::is_same<T, __nv_bfloat16>::value) {
              uint32_t* wv = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[e]));
                const __half2 h = __floats2half2_rn(f.x, f.y);  // beyond the fp16 range: +-inf
                wv[e] = *reinterpret_cast<const uint32_t*>(&h);
              }
            }
            *reinterpret_cast<uint4*>(xd + it * 16) = v;
          }
        }
        fence_proxy_async();  // generic-proxy writes, read by the tensor core
        mbar_arrive(&ofull[o]);
      }
      if (!ok || *failed) {
        *failed = 1;
        break;
      }
      mbar_arrive(&empty[s]);
    }
    if (gt == 0) *consumed = i;
  }

  // ---------------- accumulators -> rank 0 -> outputs ----------------
  const bool epi = warp >= 2 && warp <= 5;  // epilogue warps: TMEM quadrant warp % 4
  bool bad = false;
  if (epi) {
    bad = !mbar_wait(accum, 0);
    tc_fence_after();
    if (threadIdx.x == 64) STRACE(2, 0);
  }
  tc_fence_before();
  __syncthreads();
  bad = bad || *failed;
  const int q = warp & 3;
  // this lane's weight row: M = 128 accumulators use every TMEM lane, M = 64
  // ones lanes 0-15 of each 32-lane quadrant
  constexpr bool kAllLanes = FM == 128;
  const int fl = kAllLanes ? 32 * q + lane : 16 * q + lane;
  const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
  constexpr int CW = C::CW, SPAN = C::SPAN, NB = C::NB;
  const int cs = p.cs;
  const int rpo = C::rpo(cs);
  // The K split's partials meet at their owners: epilogue block j (activation
  // columns [j SPAN, (j + 1) SPAN)) belongs to rank j % cs, which receives
  // that block from the other ranks into its idle ring and finishes it.  Every
  // owner's buffer then holds only its own blocks, and every rank stores.
  float* red = reinterpret_cast<float*>(sm);
  auto load_block = [&](int c, float* g, float* u) {  // sum of the accumulator sets, columns [c, c + SPAN)
    for (int jj = 0; jj < p.na; ++jj) {
      const uint32_t tj = tq + jj * C::ACC;
      float g1[CW], u1[CW];
      if (GATE && MN < CW) {  // MN = 16: one 32-column load holds [gate | up]
        tmem_ld<CW>(tj, g1);
#pragma unroll
        for (int e = 0; e < MN; ++e) u1[e] = g1[MN + e];
      } else {
        tmem_ld<CW>(tj + c, g1);
        if (GATE) tmem_ld<CW>(tj + MN + c, u1);
      }
#pragma unroll
      for (int e = 0; e < CW; ++e) {
        g[e] = jj ? g[e] + g1[e] : g1[e];
        if (GATE) u[e] = jj ? u[e] + u1[e] : u1[e];
      }
    }
  };
  if (cs > 1) {
    cluster_sync();  // every rank's ring is idle
    if (epi) {
      // the loads are warp-collective; at M = 64 lanes 16-31 hold nothing and store nothing
#pragma unroll 1
      for (int j = 0; j < NB; ++j) {
        const int o = j % cs;
        if (o == rank) continue;
        float g[CW], u[CW];
        load_block(j * SPAN, g, u);
        if (kAllLanes || lane < 16) {
          const int slot = rank < o ? rank : rank - 1;
          float* dst = red + ((int64_t)slot * FM + fl) * rpo + (j / cs) * SPAN * C::NW;
#pragma unroll
          for (int e = 0; e < SPAN; e += 4) {
            st_cluster_f4(map_to_rank(dst + e, (uint32_t)o), g[e], g[e + 1], g[e + 2], g[e + 3]);
            if (GATE) st_cluster_f4(map_to_rank(dst + SPAN + e, (uint32_t)o), u[e], u[e + 1], u[e + 2], u[e + 3]);
          }
        }
      }
      if (bad && threadIdx.x == 64) {
        const int one = 1;
        for (int o = 0; o < cs; ++o)
          if (o != rank)
            asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(map_to_rank(peer_failed, (uint32_t)o)), "r"(one)
                         : "memory");
      }
    }
    cluster_sync();  // partials landed
  }
  if (epi) {
    bad = bad || *reinterpret_cast<volatile int*>(peer_failed);
    const int f = f0 + fl;
    const bool live = (kAllLanes || lane < 16) && f < p.N;
    const float sc0 = (live && p.s0) ? p.s0[f] : 1.f;
    const float sc1 = (live && GATE && p.s1) ? p.s1[f] : 1.f;
    T* ycol = static_cast<T*>(p.y) + f;
#pragma unroll 1
    for (int j = rank; j < NB; j += cs) {  // the blocks this rank owns (all of them without a cluster)
      const int c = j * SPAN;
      float g[CW], u[CW];
      load_block(c, g, u);
      if (live) {
        for (int r = 0; r + 1 < cs; ++r) {
          const float* src = red + ((int64_t)r * FM + fl) * rpo + (j / cs) * SPAN * C::NW;
#pragma unroll
          for (int e = 0; e < SPAN; e += 4) {
            const float4 a = *reinterpret_cast<const float4*>(src + e);
            g[e] += a.x; g[e + 1] += a.y; g[e + 2] += a.z; g[e + 3] += a.w;
            if (GATE) {
              const float4 b = *reinterpret_cast<const float4*>(src + SPAN + e);
              u[e] += b.x; u[e + 1] += b.y; u[e + 2] += b.z; u[e + 3] += b.w;
            }
          }
        }
#pragma unroll
        for (int e = 0; e < SPAN; ++e) {
          const int m = m0 + c + e;
          if (m < p.M) {
            float v = GATE ? silu_mul(g[e] * sc0, u[e] * sc1) : g[e] * sc0;
            if (bad) v = __int_as_float(0x7fc00000);
            ycol[(int64_t)m * p.ldy] = from_f<T>(v);
          }
        }
      }
    }
  }

  if (threadIdx.x == 64) STRACE(2, 1);
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *failed) {
    // copies issued but never consumed still target this CTA's shared memory
    for (int i = *consumed; i < *issued; ++i) mbar_wait(&full[i % ns], (uint32_t)((i / ns) & 1));
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

template <typename T>
constexpr CUtensorMapDataType map_dtype() {
  return std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// How many clusters of `cs` CTAs of this kernel with `smem` bytes can be
// resident at once (cached per device, ring budget and cluster size).
template <typename K>
long max_clusters(K kern, int cs, size_t smem, int budget_idx) {
  static int cache[64][2][9] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= 64 || cs < 1 || cs > 8) return 0;
  int& slot = cache[dev][budget_idx][cs];
  if (slot == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs * 64);
    cfg.blockDim = dim3(kThr);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();  // clear it: the caller then keeps K unsplit
      n = -1;
    }
    slot = n;
  }
  return slot;
}

// Operand maps: 3-D [K / 64][rows][64] views when K is a multiple of 64 (one
// TMA instruction then fetches `kc` chunks), else 2-D [rows][K] with the K
// tail zero-filled (kc == 1).
bool operand_map(CUtensorMap* m, CUtensorMapDataType dt, uint32_t esz, const void* base, int64_t K, int64_t rows,
                 int64_t ld, uint32_t box_rows, int kc, bool map3d, CUtensorMapSwizzle sw) {
  if (map3d)
    return make_map_3d(m, dt, base, BK, (uint64_t)rows, (uint64_t)(K / BK), (uint64_t)ld * esz, BK * esz, BK,
                       box_rows, (uint32_t)kc, sw);
  return make_map_2d(m, dt, base, (uint64_t)K, (uint64_t)rows, (uint64_t)ld * esz, BK, box_rows, sw);
}

template <typename T, int MN, bool GATE, bool W8>
int launch_cfg(const DenseArgs& a) {
  using C = SwapCfg<MN, GATE, W8>;
  constexpr int FM = C::FM;
  const int kchunks = (a.K + BK - 1) / BK;
  const bool map3d = a.K % BK == 0;
  const int tf = (a.N + FM - 1) / FM, tm = (a.M + MN - 1) / MN;
  const long base = (long)tf * tm;
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return B200MM_ERR_DEVICE;
  const int sms = num_sms(dev);
  // ring: one CTA per SM when the tiles fit in one wave that way, else two
  int budget_idx = base <= sms ? 0 : 1;
#ifdef SWAP_TRACE
  if (const char* e = getenv("B200MM_SWAP_BUDGET")) budget_idx = atoi(e) ? 1 : 0;
#endif
  if (budget_idx == 1 && kBudget2 < C::OPS * C::OPST + 2 * C::CHUNK) budget_idx = 0;  // big int8 tiles
  const uint32_t budget = (budget_idx == 0 ? kBudget1 : kBudget2) - C::OPS * C::OPST;
  // K-chunks per stage (a stage costs one tcgen05.commit, which stalls the
  // issuer): int8, as many as leave three stages, up to 8 (the converter
  // ring sits between the stages and the MMAs); 16-bit, as many as leave two
  // stages, up to 4 (measured: 4 chunks in 2 stages beat 2 chunks in 5 by
  // 4-9 % at M = 16..64, and gate-up 2 chunks in 2 stages beat 1 in 5 by 15 %)
  int kc = 1;
  constexpr int kMaxKc = W8 ? 8 : 4, kMinStages = W8 ? 3 : 2;
  if (map3d)
    for (int c = kMaxKc; c >= 2; c >>= 1)
      if (kchunks >= c && budget / (c * C::CHUNK) >= (uint32_t)kMinStages) {
        kc = c;
        break;
      }
#ifdef SWAP_TRACE
  if (const char* e = getenv("B200MM_SWAP_KC")) kc = map3d ? atoi(e) : 1;
#endif
  const int nstages = (kchunks + kc - 1) / kc;
  const uint32_t stage = kc * C::CHUNK;
  int ns = (int)(budget / stage);
  if (ns > kMaxNS) ns = kMaxNS;
  if (ns > nstages) ns = nstages < 2 ? 2 : nstages;
  if (ns < 2 || (uint32_t)ns * stage > budget) return B200MM_ERR_SHAPE;
  const size_t smem = (size_t)ns * stage + C::OPS * C::OPST + C::EXTRA;
  CUtensorMap mx, mw0, mw1;
  const CUtensorMapDataType dt = map_dtype<T>();
  if (!operand_map(&mx, dt, 2, a.x, a.K, a.M, a.ldx, MN, kc, map3d, CU_TENSOR_MAP_SWIZZLE_128B))
    return B200MM_ERR_ALIGN;
  const CUtensorMapDataType wdt = W8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : dt;
  const uint32_t wsz = W8 ? 1 : 2;
  const CUtensorMapSwizzle wsw = W8 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B;
  if (!operand_map(&mw0, wdt, wsz, a.w0, a.K, a.N, a.ldw0, FM, kc, map3d, wsw)) return B200MM_ERR_ALIGN;
  if (GATE) {
    if (!operand_map(&mw1, wdt, wsz, a.w1, a.K, a.N, a.ldw1, FM, kc, map3d, wsw)) return B200MM_ERR_ALIGN;
  } else {
    mw1 = mw0;
  }
  auto kern = tc_swap_kernel<T, MN, GATE, W8>;
  static bool configured[64] = {false};
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kBudget1 + C::EXTRA)) !=
        cudaSuccess)
      return B200MM_ERR_LAUNCH;
    configured[dev] = true;
  }
  // K split over a cluster while every tile's cluster is resident at once,
  // each rank keeps two stages or more, and rank 0's ring holds the partials
  const long slots = (long)sms * (budget_idx == 0 ? 1 : 2);
  int cs = 1, cs_cap = 8;
#ifdef SWAP_TRACE
  if (const char* e = getenv("B200MM_SWAP_CS")) cs_cap = atoi(e);
#endif
  for (int c = 2; c <= cs_cap && c <= nstages / 2 && base * c <= slots && C::red_bytes(c) <= ns * stage;
       ++c) {
    if (base > max_clusters(kern, c, smem, budget_idx)) break;
    cs = c;
  }
  if ((long)tf * cs > 2147483647L || tm > 65535) return B200MM_ERR_SHAPE;
  // accumulator sets: up to one per K step of a chunk, within this CTA's
  // share of TMEM
  const int tmem_share = budget_idx == 0 ? 512 : 256;
  int na = 4;
  while (na > 1 && na * C::ACC > tmem_share) na >>= 1;
  const int cols = na * C::ACC;
  const uint32_t tmem_cols = cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
  SwapParams p{a.s0, a.s1, a.y, a.ldy, a.M, a.N, a.K, nstages, kc, map3d ? 1 : 0, ns, cs, na, tmem_cols, 0};
#ifdef SWAP_TRACE
  if (const char* d = getenv("B200MM_SWAP_DEBUG")) p.debug = atoi(d);
#endif
  const dim3 grid((unsigned)(tf * cs), (unsigned)tm);
  const cudaError_t e = cs > 1 ? launch_pdl_cluster(kern, grid, dim3(kThr), smem, a.stream, cs, mx, mw0, mw1, p)
                               : launch_pdl(kern, grid, dim3(kThr), smem, a.stream, mx, mw0, mw1, p);
  return e == cudaSuccess ? B200MM_OK : B200MM_ERR_LAUNCH;
}

template <typename T, bool GATE, bool W8>
int launch_mn(const DenseArgs& a) {
  if (a.M <= 16) return launch_cfg<T, 16, GATE, W8>(a);
  if (a.M <= 32) return launch_cfg<T, 32, GATE, W8>(a);
  if (a.M <= 64) return launch_cfg<T, 64, GATE, W8>(a);
  if (a.M <= 128) return launch_cfg<T, 128, GATE, W8>(a);
  return launch_cfg<T, 256, GATE, W8>(a);
}

template <typename T>
int launch_t(const DenseArgs& a) {
  if (a.w8) return a.gate ? launch_mn<T, true, true>(a) : launch_mn<T, false, true>(a);
  return a.gate ? launch_mn<T, true, false>(a) : launch_mn<T, false, false>(a);
}

}  // namespace

#ifdef SWAP_TRACE
extern "C" int b200mm_debug_trace(void* host, size_t bytes) {
  return cudaMemcpyFromSymbol(host, g_swap_trace, bytes < sizeof(g_swap_trace) ? bytes : sizeof(g_swap_trace)) ==
                 cudaSuccess
             ? 0
             : 1;
}
#endif

bool swap_supported(const DenseArgs& a) {
  if (a.dtype != B200MM_BF16 && a.dtype != B200MM_F16) return false;
  if (a.M < 5) return false;
  const int wsz = a.w8 ? 1 : 2;
  if (!al16(a.x) || !al16(a.w0) || (a.gate && !al16(a.w1))) return false;
  if ((a.ldx * 2) % 16 || (a.ldw0 * wsz) % 16 || (a.gate && (a.ldw1 * wsz) % 16)) return false;
  if ((a.K * 2) % 16 || (a.K * wsz) % 16) return false;
  return true;
}

int swap_launch(const DenseArgs& a) {
  if (a.dtype == B200MM_BF16) return launch_t<__nv_bfloat16>(a);
  return launch_t<__half>(a);
}

}  // namespace b200mm
