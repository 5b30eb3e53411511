// Small-M (decode) projection kernel: weight-streaming GEMV for M <= 8.
//
// The weight matrix is the only large operand (31.5 MB for the Qwen3-4B QKV
// projection, 99.6 MB for gate+up), so the kernel is an HBM stream:
//   * every warp owns a "unit" of two weight rows (gate row n + up row n for
//     the gate-up epilogue, rows 2u and 2u+1 for QKV) and reads both rows end
//     to end with 16-byte, L1-bypassing loads -- NCH loads per lane per row in
//     flight before the first FMA;
//   * the activation rows x[0..M) are staged once per CTA in shared memory in
//     their own dtype, so one 16-byte shared load feeds both weight rows;
//   * fp32 accumulation, warp-shuffle reduction, and the SiLU*up / int8 scale
//     epilogue in registers: the [M, 2N] gate/up intermediate never exists;
//   * launched with programmatic dependent launch: a warp issues the loads of
//     its first unit's weights before `griddepcontrol.wait`, so weight
//     streaming overlaps the tail of the kernel that produced x.
//   * shapes with fewer units than resident warps (column shards, narrow
//     projections) split each unit's K range over 2-8 warps of a CTA, which
//     sum their partials through shared memory.
// Grid: (SM count) x (resident CTAs per SM), grid-stride over units.
#include "dense.cuh"

namespace b200mm {

namespace {

constexpr int kThreads = 256;

struct GemvParams {
  const void* x; int64_t ldx;
  const void* w0; int64_t ldw0;
  const void* w1; int64_t ldw1;
  const float* s0; const float* s1;
  void* y; int64_t ldy;
  int M, N, K;
};

// The peer-output block is a kernel parameter of the general form only: in
// the plain form it is an empty struct, so the plain launches carry the
// original ~100-byte parameter block.
template <bool GEN> struct PeerArg { int world; };  // plain: never peer output (world = 0)
template <> struct PeerArg<true> : PeerEpi {};

// Two CTAs per SM for M <= 4 (at most 128 registers).  Three per SM with
// fewer loads in flight made a lone QKV launch faster, but in the decode step
// the QKV and gate-up launches alternate and a register-full QKV grid keeps
// the next gate-up grid from starting early, which cost more than it saved.
template <int MR, bool GATE>
constexpr int gemv_min_blocks() {
  return MR <= 4 ? 2 : 1;
}

// GEN: the general form (K slices, peer output); the plain form compiles
// both out (ks = 1, local y), since the general form's extra state cost the
// whole-shape QKV launch ~5 % (7.0 -> 7.4 us).
template <typename TX, typename TW, int MR, bool GATE, int NCH, bool GEN>
__global__ void __launch_bounds__(kThreads, gemv_min_blocks<MR, GATE>())
gemv_kernel(const GemvParams p, const int nsm, const int ks_arg, const PeerArg<GEN> pe) {
  const int ks = GEN ? ks_arg : 1;
  const int world = GEN ? pe.world : 0;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TX* xs = reinterpret_cast<TX*>(smem_raw);  // [MR][K] activation rows
  __shared__ float red[kThreads / 32][2][MR];  // K-slice partial sums (ks > 1)

  constexpr int WV = Chunk<TW>::kElems;      // weights per 16-byte chunk
  constexpr int XV = Chunk<TX>::kElems;      // activations per 16-byte chunk
  static_assert(WV % XV == 0, "weight chunk must cover whole activation chunks");
  constexpr int XPW = WV / XV;               // activation chunks per weight chunk

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps_per_cta = blockDim.x >> 5;
  const int N = p.N, K = p.K, M = p.M;
  const int nunits = GATE ? N : (N + 1) >> 1;
  const int nchunks = K / WV;
  constexpr int kSeg = 32 * NCH;

  // Work items.  ks == 1: a warp owns whole units, grid-stride.  Unit order:
  // block order (gate-up): warp w of CTA b takes units b * warps + w + k *
  // nwarps.  SM-round-robin order (plain projections, nsm > 0, the grid a
  // multiple of the SM count so CTA b runs on SM b % nsm): consecutive units
  // go to consecutive SMs, so the last, partial wave of units is spread over
  // every SM instead of the first CTAs' SMs.  Measured (Qwen3-4B QKV, M = 1,
  // 36 launches in a graph): 7.8 -> 6.9 us; for gate-up it was slower (17.4
  // -> 17.9 us) and stays in block order.
  // ks > 1 (too few units to give every warp one: column shards, narrow
  // projections): the ks warps of a group split one unit's K range and sum
  // their partials through shared memory; a CTA takes warps / ks units at a
  // time, grid-stride, every warp of the CTA in step (the sums need
  // __syncthreads).
  const int upc = warps_per_cta / ks;  // units per CTA tile
  const int slice = warp % ks;
  const int cps = (nchunks + ks - 1) / ks;  // chunks per K slice
  const int cbeg = slice * cps;
  const int cend = cbeg + cps < nchunks ? cbeg + cps : nchunks;
  const int nseg = (cend - cbeg + kSeg - 1) / kSeg;
  int u, ustep;
  if (ks == 1) {
    u = blockIdx.x * warps_per_cta + warp;
    if (nsm > 0 && gridDim.x % nsm == 0)
      u = ((int)(blockIdx.x / nsm) * warps_per_cta + warp) * nsm + blockIdx.x % nsm;
    ustep = gridDim.x * warps_per_cta;
  } else {
    u = blockIdx.x * upc + warp / ks;
    ustep = gridDim.x * upc;
  }
  // ks > 1: every warp runs the tile loop while its CTA has a tile
  const int ntile_units = ks == 1 ? nunits : ((nunits + upc - 1) / upc) * upc;

  const TW* w0 = static_cast<const TW*>(p.w0);
  const TW* w1 = static_cast<const TW*>(p.w1);

  auto row_ptrs = [&](int uu, const TW*& r0, const TW*& r1, bool& v1) {
    if (GATE) {
      r0 = w0 + (int64_t)uu * p.ldw0;
      r1 = w1 + (int64_t)uu * p.ldw1;
      v1 = true;
    } else {
      const int n0 = 2 * uu;
      r0 = w0 + (int64_t)n0 * p.ldw0;
      v1 = (n0 + 1) < N;
      r1 = w0 + (int64_t)(v1 ? n0 + 1 : n0) * p.ldw0;
    }
  };

  uint4 wv[2][NCH];
  auto load_seg = [&](int uu, int seg) {
    const TW* r0; const TW* r1; bool v1;
    row_ptrs(uu, r0, r1, v1);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int c = cbeg + seg * kSeg + i * 32 + lane;
      if (c < cend) {
        wv[0][i] = ld_stream16(r0 + (int64_t)c * WV);
        wv[1][i] = v1 ? ld_stream16(r1 + (int64_t)c * WV) : make_uint4(0, 0, 0, 0);
      } else {
        wv[0][i] = make_uint4(0, 0, 0, 0);
        wv[1][i] = make_uint4(0, 0, 0, 0);
      }
    }
  };

  // int8 weights: the warp's next unit is pulled into L2 while this one is
  // computed (the registers bound the loads in flight, L2 prefetches are free
  // of them; int8 units are half the bytes, so a warp walks twice as many).
  // Measured: int8 QKV 11.5 -> 10.3 us, gate-up 26.7 -> 25.1 us at M = 1;
  // for 16-bit weights it slowed both (gate-up 17.3 -> 18.9 us), so it is off.
  auto prefetch_unit = [&](int un) {
    const TW* r0; const TW* r1; bool v1;
    row_ptrs(un, r0, r1, v1);
    const char* p0 = reinterpret_cast<const char*>(r0 + (int64_t)cbeg * WV);
    const char* p1 = reinterpret_cast<const char*>(r1 + (int64_t)cbeg * WV);
    const int64_t bytes = (int64_t)(cend - cbeg) * 16;
    for (int64_t off = (int64_t)lane * 128; off < bytes; off += 32 * 128) {
      prefetch_l2(p0 + off);
      if (v1) prefetch_l2(p1 + off);
    }
  };

  // Weights are never written by another kernel: start streaming them now.
  if (u < nunits) load_seg(u, 0);
  pdl_trigger();
  pdl_wait();

  // Stage x[0..M) (zero rows M..MR) in shared memory, 16 bytes at a time.
  {
    const TX* x = static_cast<const TX*>(p.x);
    const int kc = K / XV;  // 16-byte chunks per row
    for (int i = threadIdx.x; i < MR * kc; i += blockDim.x) {
      const int m = i / kc, c = i - m * kc;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (m < M) v = *reinterpret_cast<const uint4*>(x + (int64_t)m * p.ldx + (int64_t)c * XV);
      *reinterpret_cast<uint4*>(xs + (int64_t)m * K + (int64_t)c * XV) = v;
    }
  }
  __syncthreads();

  bool preloaded = true;
  for (; u < ntile_units; u += ustep) {
    const bool live = u < nunits;
    if (sizeof(TW) == 1 && live && u + ustep < nunits) prefetch_unit(u + ustep);
    float acc[2][MR];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int m = 0; m < MR; ++m) acc[r][m] = 0.f;

    for (int seg = 0; live && seg < nseg; ++seg) {
      if (!preloaded) load_seg(u, seg);
      preloaded = false;
#pragma unroll
      for (int i = 0; i < NCH; ++i) {
        const int c = cbeg + seg * kSeg + i * 32 + lane;
        if (c < cend) {
          float f0[WV], f1[WV];
          Chunk<TW>::unpack(wv[0][i], f0);
          Chunk<TW>::unpack(wv[1][i], f1);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            const TX* xp = xs + (int64_t)m * K + (int64_t)c * WV;
#pragma unroll
            for (int h = 0; h < XPW; ++h) {
              float xf[XV];
              Chunk<TX>::unpack(*reinterpret_cast<const uint4*>(xp + h * XV), xf);
#pragma unroll
              for (int e = 0; e < XV; ++e) {
                acc[0][m] = fmaf(f0[h * XV + e], xf[e], acc[0][m]);
                acc[1][m] = fmaf(f1[h * XV + e], xf[e], acc[1][m]);
              }
            }
          }
        }
      }
    }
    preloaded = false;

#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int m = 0; m < MR; ++m) acc[r][m] = warp_sum(acc[r][m]);

    if (ks > 1) {
      // the group's slices meet in shared memory; slice 0 stores
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int m = 0; m < MR; ++m) red[warp][r][m] = acc[r][m];
      }
      __syncthreads();
      if (slice == 0) {
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            float t = 0.f;
            for (int s = 0; s < ks; ++s) t += red[warp + s][r][m];
            acc[r][m] = t;
          }
      }
      __syncthreads();
    }

    // lanes 0..MR-1 store row m = lane (values are uniform across the warp)
    if (live && slice == 0 && lane < MR && lane < M) {
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int m = 0; m < MR; ++m)
        if (m == lane) { a0 = acc[0][m]; a1 = acc[1][m]; }
      TX* y = static_cast<TX*>(p.y) + (int64_t)lane * p.ldy;
      auto put = [&](int n, float v) {
        if (world == 0) {
          y[n] = from_f<TX>(v);
        } else {
          if constexpr (GEN) peer_store(pe, lane, n, from_f<TX>(v));
        }
      };
      if (GATE) {
        if (p.s0) { a0 *= p.s0[u]; a1 *= p.s1[u]; }
        put(u, silu_mul(a0, a1));
      } else {
        const int n0 = 2 * u;
        if (p.s0) a0 *= p.s0[n0];
        put(n0, a0);
        if (n0 + 1 < N) {
          if (p.s0) a1 *= p.s0[n0 + 1];
          put(n0 + 1, a1);
        }
      }
    }
  }
  if constexpr (GEN) {
    if (world > 0) peer_finish(pe);
  }
}

template <typename TX, typename TW, int MR, bool GATE>
int launch_one(const DenseArgs& a) {
  constexpr int NCH = (sizeof(TW) == 2) ? 10 : 8;
  auto kplain = gemv_kernel<TX, TW, MR, GATE, NCH, false>;
  auto kgen = gemv_kernel<TX, TW, MR, GATE, NCH, true>;
  const size_t smem = (size_t)MR * a.K * sizeof(TX);
  static int configured_smem[2][64] = {{0}};  // per form and device: largest opt-in set so far
  static int blocks_per_sm[2][64][8] = {{{0}}};
  int dev = current_device();
  if (dev < 0 || dev >= 64) return B200MM_ERR_DEVICE;
  // occupancy depends on smem; cache per (form, device, smem bucket of 32 KB)
  const int bucket = (int)(smem >> 15) < 8 ? (int)(smem >> 15) : 7;
  auto prepare = [&](int g, auto kern) -> int {
    if (smem > 48 * 1024 && (int)smem > configured_smem[g][dev]) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return -1;
      configured_smem[g][dev] = (int)smem;
    }
    int& b = blocks_per_sm[g][dev][bucket];
    if (b == 0) {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, kThreads, smem) != cudaSuccess || b < 1)
        b = 1;
    }
    return b;
  };
  int bps = prepare(0, kplain);
  if (bps < 0) return B200MM_ERR_LAUNCH;
  const int nunits = a.gate ? a.N : (a.N + 1) / 2;
  const int warps_per_cta = kThreads / 32;
  const int slots = num_sms(dev) * bps * warps_per_cta;  // resident warps
  // K slices per unit: the most (1, 2, 4, 8) that keep every (unit, slice)
  // in one wave of resident warps, each slice keeping at least one 16-byte
  // chunk per lane.  Measured at M = 1 (graphs of launches, weights past L2):
  // a QKV column shard of 768 rows 3.05 -> 2.71 us, 1536 rows 3.31 -> 3.16,
  // a 320-row o shard 4.51 -> 2.51; slicing shapes that already fill one wave
  // (the whole QKV, gate-up) made them 25-40 % slower, so they keep ks = 1.
  constexpr int WV = 16 / (int)sizeof(TW);
  int ks = 1;
  while (ks < 8 && (int64_t)nunits * 2 * ks <= slots && a.K / WV / (2 * ks) >= 32) ks *= 2;
  const int gen = ks > 1 || a.peer ? 1 : 0;
  if (gen) {
    bps = prepare(1, kgen);
    if (bps < 0) return B200MM_ERR_LAUNCH;
  }
  const int upc = warps_per_cta / ks;
  int grid = num_sms(dev) * bps;
  const int need = (nunits + upc - 1) / upc;
  if (grid > need) grid = need;
  if (grid < 1) grid = 1;
  GemvParams p{a.x, a.ldx, a.w0, a.ldw0, a.w1, a.ldw1, a.s0, a.s1, a.y, a.ldy, a.M, a.N, a.K};
  PeerArg<true> pe{};
  if (a.peer) peer_epi_from(*a.peer, pe);
  // plain projections: warps take units in SM-round-robin order (below)
  const int order = GATE ? 0 : num_sms(dev);
  cudaError_t e = gen ? launch_pdl(kgen, dim3(grid), dim3(kThreads), smem, a.stream, p, order, ks, pe)
                      : launch_pdl(kplain, dim3(grid), dim3(kThreads), smem, a.stream, p, order, ks, PeerArg<false>{0});
  return e == cudaSuccess ? B200MM_OK : B200MM_ERR_LAUNCH;
}

template <typename TX, typename TW, bool GATE>
int launch_mr(const DenseArgs& a) {
  if (a.M <= 1) return launch_one<TX, TW, 1, GATE>(a);
  if (a.M <= 2) return launch_one<TX, TW, 2, GATE>(a);
  if (a.M <= 4) return launch_one<TX, TW, 4, GATE>(a);
  return launch_one<TX, TW, 8, GATE>(a);
}

template <typename TX, typename TW>
int launch_gate(const DenseArgs& a) {
  return a.gate ? launch_mr<TX, TW, true>(a) : launch_mr<TX, TW, false>(a);
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

bool gemv_supported(const DenseArgs& a) {
  if (a.M < 1 || a.M > 8) return false;
  const int xsz = a.dtype == B200MM_F32 ? 4 : 2;
  const int wsz = a.w8 ? 1 : xsz;
  const int wv = 16 / wsz;
  if (a.K % wv != 0) return false;
  if ((a.K * xsz) % 16 != 0) return false;
  if (!aligned16(a.x) || (a.ldx * xsz) % 16 != 0) return false;
  if (!aligned16(a.w0) || (a.ldw0 * wsz) % 16 != 0) return false;
  if (a.gate && (!aligned16(a.w1) || (a.ldw1 * wsz) % 16 != 0)) return false;
  const int mr = a.M <= 1 ? 1 : a.M <= 2 ? 2 : a.M <= 4 ? 4 : 8;
  if ((size_t)mr * a.K * xsz > 200 * 1024) return false;
  return true;
}

int gemv_launch(const DenseArgs& a) {
  if (a.w8) {
    if (a.dtype == B200MM_BF16) return launch_gate<__nv_bfloat16, int8_t>(a);
    if (a.dtype == B200MM_F16) return launch_gate<__half, int8_t>(a);
    return B200MM_ERR_DTYPE;
  }
  if (a.dtype == B200MM_BF16) return launch_gate<__nv_bfloat16, __nv_bfloat16>(a);
  if (a.dtype == B200MM_F16) return launch_gate<__half, __half>(a);
  if (a.dtype == B200MM_F32) return launch_gate<float, float>(a);
  return B200MM_ERR_DTYPE;
}

}  // namespace b200mm
