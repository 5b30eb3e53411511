// Mid-M projection kernel (5 <= M <= 64): weight-streaming tensor-core GEMV.
//
// Still an HBM stream (the weights dominate the bytes up to M ~ 128), but with
// M activation rows the CUDA-core GEMV would need M FMAs per weight element,
// so the products run on mma.sync m16n8k16 instead:
//   * weights are the A operand (16 weight rows per warp), read straight from
//     HBM into A fragments: lane l loads 16 bytes of rows l/4 and l/4 + 8 at
//     k offset 8*(l%4) (16 for int8) and splits them across consecutive
//     k16 MMAs.  That permutes K inside each 32-column (64 for int8) chunk;
//     the activations (the B operand) are read with the same permutation, so
//     every dot product is unchanged;
//   * activations x[M, K-slice] are staged once per CTA in shared memory
//     (padded rows, conflict-free 16-byte loads), in the MMA input dtype;
//   * int8 weights become fp16 exactly (|q| <= 127): the byte, sign-flipped,
//     is spliced under the fp16 exponent of 1024 by one byte-permute and
//     1152 is subtracted from the pair; x is then staged as fp16
//     (satfinite conversion: |x| beyond 65504 saturates);
//   * K is split over a cluster of CS = 4 or 8 CTAs (each owns 1/CS of K for
//     the same 128 weight rows); the partial sums meet through distributed
//     shared memory: CTA r receives the partials of rows [r*128/CS, +128/CS)
//     from all CS ranks and finishes them (int8 scale, SiLU * up), so there
//     is no workspace and no atomic.  CS = 8 when four-way groups would not
//     fill the SMs (narrow outputs such as the 2560-row o / down
//     projections);
//   * launched with programmatic dependent launch; a warp issues its first
//     weight loads before griddepcontrol.wait.
#include <cstdlib>
#include <type_traits>

#include "dense.cuh"

namespace b200mm {

namespace {

constexpr int kWarps = 8;            // 8 x 16 = 128 weight rows per CTA
constexpr int kThreads = 32 * kWarps;
constexpr int kRows = 16 * kWarps;   // weight rows per CTA (per matrix)

struct MmvParams {
  const void* x; int64_t ldx;
  const void* w0; int64_t ldw0;
  const void* w1; int64_t ldw1;
  const float* s0; const float* s1;
  void* y; int64_t ldy;
  int M, N, K;
  int kslice;  // K columns per cluster rank (multiple of 64)
};

// The peer-output block is a kernel parameter of the peer form only (an
// empty struct otherwise): the larger parameter block slowed the plain
// launches (8B int8 QKV at M = 4: 9.8 -> 11.0 us).
template <bool PEER> struct MmvPeer { int world; };
template <> struct MmvPeer<true> : PeerEpi {};

template <typename T> struct MmaOp;
template <> struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};
template <> struct MmaOp<__half> {
  __device__ __forceinline__ static void run(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

// TX: activation dtype in memory; TM: MMA input dtype (== TX, or fp16 for int8
// weights); TW: weight dtype; MT: n-tiles of 8 activation rows.
template <typename TX, typename TM, typename TW, int MT, bool GATE, int CS, bool PEER>
__global__ void __launch_bounds__(kThreads) mmv_kernel(const MmvParams p, const MmvPeer<PEER> pe) {
  constexpr bool W8 = sizeof(TW) == 1;
  constexpr int KC = W8 ? 64 : 32;       // K columns per warp-chunk (4 lanes x 16 bytes)
  constexpr int NM = GATE ? 2 : 1;
  constexpr int MP = 8 * MT;             // padded activation rows
  // chunks in flight per warp (measured): a 16-bit QKV chunk is only 1 KB per
  // warp, so QKV keeps 8 (int8: 4 up to 16 rows); gate-up holds two matrices'
  // chunks and loses occupancy beyond 2
  constexpr int U = GATE ? 2 : (W8 ? (MT <= 2 ? 4 : 2) : 8);
  constexpr int RP = MP + 2;             // reduction row pitch: even, so float2 stores stay aligned
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // row pitch (elements): a 16-byte load phase of 8 lanes covers 2 rows x 64
  // bytes (16-bit weights) or 4 rows x 32 bytes (int8); rows shift by 64 / 16 bytes
  const int xpitch = p.kslice + (W8 ? 8 : 32);
  TM* xs = reinterpret_cast<TM*>(smem_raw);                                            // [MP][xpitch]
  constexpr int RPO = kRows / CS;       // rows finished per cluster rank
  float* red = reinterpret_cast<float*>(smem_raw + (size_t)MP * xpitch * sizeof(TM));  // [NM][CS][RPO][RP]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t rank = cluster_rank();
  const int group = blockIdx.x / CS;
  const int row_base = group * kRows + 16 * warp;   // this warp's 16 weight rows
  const int k_begin = (int)rank * p.kslice;
  const int k_end = min(p.K, k_begin + p.kslice);
  const int nchunks = k_end > k_begin ? (k_end - k_begin + KC - 1) / KC : 0;
  const int r_lo = row_base + (lane >> 2), r_hi = r_lo + 8;
  const bool v_lo = r_lo < p.N, v_hi = r_hi < p.N;
  const int lk = (lane & 3) * (W8 ? 16 : 8);        // this lane's k offset inside a chunk

  const TW* wp[NM][2];
#pragma unroll
  for (int mtx = 0; mtx < NM; ++mtx) {
    const TW* base = static_cast<const TW*>(mtx ? p.w1 : p.w0);
    const int64_t ld = mtx ? p.ldw1 : p.ldw0;
    wp[mtx][0] = base + (int64_t)(v_lo ? r_lo : 0) * ld;
    wp[mtx][1] = base + (int64_t)(v_hi ? r_hi : 0) * ld;
  }
  auto ld_chunk = [&](int c, int mtx, int h) -> uint4 {
    const int kk = k_begin + c * KC + lk;
    const bool ok = (h ? v_hi : v_lo) && kk < k_end;
    return ok ? ld_stream16(wp[mtx][h] + kk) : make_uint4(0, 0, 0, 0);
  };

  // weights are never written by the previous kernel: start streaming them now
  uint4 wv[U][NM][2];
#pragma unroll
  for (int u = 0; u < U; ++u)
#pragma unroll
    for (int mtx = 0; mtx < NM; ++mtx)
#pragma unroll
      for (int h = 0; h < 2; ++h) wv[u][mtx][h] = u < nchunks ? ld_chunk(u, mtx, h) : make_uint4(0, 0, 0, 0);

  pdl_trigger();
  pdl_wait();

  // stage x[:, k_begin:k_end) (rows >= M and columns >= k_end as zero)
  {
    const TX* x = static_cast<const TX*>(p.x);
    const int w2 = p.kslice / 2;
    for (int i = threadIdx.x; i < MP * w2; i += kThreads) {
      const int m = i / w2, kp = 2 * (i - m * w2);
      const int k = k_begin + kp;
      float a = 0.f, b = 0.f;
      if (m < p.M) {
        if (k < k_end) a = to_f<TX>(x[(int64_t)m * p.ldx + k]);
        if (k + 1 < k_end) b = to_f<TX>(x[(int64_t)m * p.ldx + k + 1]);
      }
      uint32_t v;
      if constexpr (std::is_same<TM, __half>::value) {
        asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(v) : "f"(b), "f"(a));  // a -> low half
      } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        v = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint32_t*>(xs + (int64_t)m * xpitch + kp) = v;
    }
  }
  __syncthreads();

  float acc[NM][MT][4];
#pragma unroll
  for (int mtx = 0; mtx < NM; ++mtx)
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mtx][t][e] = 0.f;

  const TM* xl = xs + (int64_t)(lane >> 2) * xpitch + lk;  // this lane's activation row (n-tile 0)
  for (int c0 = 0; c0 < nchunks; c0 += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u;
      if (c < nchunks) {
        // activation fragments: 16 bytes per n-tile (32 for int8), same K permutation as the weights
        uint4 xa[MT], xb[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const TM* xr = xl + (int64_t)(8 * t) * xpitch + c * KC;
          xa[t] = *reinterpret_cast<const uint4*>(xr);
          if (W8) xb[t] = *reinterpret_cast<const uint4*>(xr + 8);
        }
#pragma unroll
        for (int mtx = 0; mtx < NM; ++mtx) {
          const uint4 lo = wv[u][mtx][0], hi = wv[u][mtx][1];
          if constexpr (!W8) {
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              MmaOp<TM>::run(acc[mtx][t], lo.x, hi.x, lo.y, hi.y, xa[t].x, xa[t].y);
              MmaOp<TM>::run(acc[mtx][t], lo.z, hi.z, lo.w, hi.w, xa[t].z, xa[t].w);
            }
          } else {
            const uint32_t L[4] = {lo.x ^ 0x80808080u, lo.y ^ 0x80808080u, lo.z ^ 0x80808080u, lo.w ^ 0x80808080u};
            const uint32_t H[4] = {hi.x ^ 0x80808080u, hi.y ^ 0x80808080u, hi.z ^ 0x80808080u, hi.w ^ 0x80808080u};
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // MMA q: word q of each row (4 k = pairs 2q, 2q+1)
              const uint32_t a0 = i8x2_to_h2(L[q], 0), a2 = i8x2_to_h2(L[q], 1);
              const uint32_t a1 = i8x2_to_h2(H[q], 0), a3 = i8x2_to_h2(H[q], 1);
#pragma unroll
              for (int t = 0; t < MT; ++t) {
                const uint32_t b0 = q < 2 ? (q == 0 ? xa[t].x : xa[t].z) : (q == 2 ? xb[t].x : xb[t].z);
                const uint32_t b1 = q < 2 ? (q == 0 ? xa[t].y : xa[t].w) : (q == 2 ? xb[t].y : xb[t].w);
                MmaOp<TM>::run(acc[mtx][t], a0, a1, a2, a3, b0, b1);
              }
            }
          }
        }
        // refill this slot with chunk c + U
#pragma unroll
        for (int mtx = 0; mtx < NM; ++mtx)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            wv[u][mtx][h] = c + U < nchunks ? ld_chunk(c + U, mtx, h) : make_uint4(0, 0, 0, 0);
      }
    }
  }

  // partials -> owner CTA (cluster rank = local row / RPO) through distributed shared memory
  {
    const int owner = (16 * warp) / RPO;
    const int lrow = (16 * warp) % RPO + (lane >> 2);
#pragma unroll
    for (int mtx = 0; mtx < NM; ++mtx)
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          float* dst = red + ((int64_t)(mtx * CS + rank) * RPO + lrow + 8 * hf) * RP + 8 * t + 2 * (lane & 3);
          st_cluster_f2(map_to_rank(dst, (uint32_t)owner), acc[mtx][t][2 * hf], acc[mtx][t][2 * hf + 1]);
        }
  }
  cluster_sync();

  // finish rows [RPO*rank, +RPO) of this group: sum the CS K-slices, epilogue, store
  {
    TX* y = static_cast<TX*>(p.y);
    for (int i = threadIdx.x; i < RPO * p.M; i += kThreads) {
      const int m = i / RPO, lr = i % RPO;
      const int n = group * kRows + RPO * (int)rank + lr;
      if (n >= p.N) continue;
      float v[NM];
#pragma unroll
      for (int mtx = 0; mtx < NM; ++mtx) {
        float s = 0.f;
#pragma unroll
        for (int r = 0; r < CS; ++r) s += red[((int64_t)(mtx * CS + r) * RPO + lr) * RP + m];
        v[mtx] = s;
      }
      float out;
      if (GATE) {
        float g = v[0], u = v[NM - 1];
        if (p.s0) { g *= p.s0[n]; u *= p.s1[n]; }
        out = silu_mul(g, u);
      } else {
        out = v[0];
        if (p.s0) out *= p.s0[n];
      }
      if constexpr (PEER)
        peer_store(pe, m, n, from_f<TX>(out));
      else
        y[(int64_t)m * p.ldy + n] = from_f<TX>(out);
    }
  }
  if constexpr (PEER) peer_finish(pe);
}

size_t smem_bytes(int MT, bool gate, bool w8, int kslice) {
  const int MP = 8 * MT;
  return (size_t)MP * (kslice + (w8 ? 8 : 32)) * 2 + (size_t)(gate ? 2 : 1) * kRows * (MP + 2) * sizeof(float);
}

template <typename TX, typename TM, typename TW, int MT, bool GATE, int CS>
int launch_mmv(const DenseArgs& a, int kslice) {
  auto kern = mmv_kernel<TX, TM, TW, MT, GATE, CS, false>;
  auto kpeer = mmv_kernel<TX, TM, TW, MT, GATE, CS, true>;
  const size_t smem = smem_bytes(MT, GATE, sizeof(TW) == 1, kslice);
  if (smem > 220 * 1024) return B200MM_ERR_SHAPE;
  static int configured[2][64] = {{0}};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return B200MM_ERR_DEVICE;
  auto prepare = [&](int g, auto k) -> bool {
    if ((int)smem > configured[g][dev]) {
      if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return false;
      configured[g][dev] = (int)smem;
    }
    return true;
  };
  MmvParams p{a.x, a.ldx, a.w0, a.ldw0, a.w1, a.ldw1, a.s0, a.s1, a.y, a.ldy, a.M, a.N, a.K, kslice};
  const int groups = (a.N + kRows - 1) / kRows;
  cudaError_t e;
  if (a.peer) {
    if (!prepare(1, kpeer)) return B200MM_ERR_LAUNCH;
    MmvPeer<true> pe{};
    peer_epi_from(*a.peer, pe);
    e = launch_pdl_cluster(kpeer, dim3(groups * CS), dim3(kThreads), smem, a.stream, CS, p, pe);
  } else {
    if (!prepare(0, kern)) return B200MM_ERR_LAUNCH;
    e = launch_pdl_cluster(kern, dim3(groups * CS), dim3(kThreads), smem, a.stream, CS, p, MmvPeer<false>{0});
  }
  return e == cudaSuccess ? B200MM_OK : B200MM_ERR_LAUNCH;
}

template <typename TX, typename TM, typename TW, bool GATE, int CS>
int launch_mt(const DenseArgs& a, int kslice) {
  if (a.M <= 8) return launch_mmv<TX, TM, TW, 1, GATE, CS>(a, kslice);
  if (a.M <= 16) return launch_mmv<TX, TM, TW, 2, GATE, CS>(a, kslice);
  if (a.M <= 32) return launch_mmv<TX, TM, TW, 4, GATE, CS>(a, kslice);
  return launch_mmv<TX, TM, TW, 8, GATE, CS>(a, kslice);
}

template <typename TX, typename TM, typename TW>
int launch_g(const DenseArgs& a, int cs, int kslice) {
  if (cs == 8)
    return a.gate ? launch_mt<TX, TM, TW, true, 8>(a, kslice) : launch_mt<TX, TM, TW, false, 8>(a, kslice);
  return a.gate ? launch_mt<TX, TM, TW, true, 4>(a, kslice) : launch_mt<TX, TM, TW, false, 4>(a, kslice);
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Cluster size: eight-way K split when four-way groups leave SMs idle.
int cluster_of(const DenseArgs& a) {
  const int groups = (a.N + kRows - 1) / kRows;
  int cs = groups * 4 < num_sms(current_device()) ? 8 : 4;
  // int8 weights up to 16 rows: a unit is half the bytes of a 16-bit one, so
  // the eight-way split keeps twice the CTAs streaming (measured, Qwen3-8B
  // int8 at M = 16: QKV 22.6 -> 15.7 us, gate-up 47.5 -> 45.0 us; at M = 32
  // it was slower)
  if (a.w8 && a.M <= 16) cs = 8;
#ifdef SWAP_TRACE
  if (const char* e = getenv("B200MM_MMV_CS")) cs = atoi(e) == 8 ? 8 : 4;
#endif
  return cs;
}

// K columns per cluster rank: a multiple of 64 (both chunk widths divide it)
int kslice_of(const DenseArgs& a, int cs) {
  const int per = (a.K + cs - 1) / cs;
  return (per + 63) / 64 * 64;
}

}  // namespace

bool mmv_supported(const DenseArgs& a) {
  if (a.M < 2 || a.M > 64) return false;
  if (a.dtype != B200MM_BF16 && a.dtype != B200MM_F16) return false;
  const int wsz = a.w8 ? 1 : 2;
  if (a.K % (16 / wsz)) return false;
  if (!al16(a.w0) || (a.ldw0 * wsz) % 16) return false;
  if (a.gate && (!al16(a.w1) || (a.ldw1 * wsz) % 16)) return false;
  const int MT = a.M <= 8 ? 1 : a.M <= 16 ? 2 : a.M <= 32 ? 4 : 8;
  return smem_bytes(MT, a.gate, a.w8, kslice_of(a, cluster_of(a))) <= 220 * 1024;
}

int mmv_launch(const DenseArgs& a) {
  const int cs = cluster_of(a);
  const int ks = kslice_of(a, cs);
  if (a.w8) {
    if (a.dtype == B200MM_BF16) return launch_g<__nv_bfloat16, __half, int8_t>(a, cs, ks);
    return launch_g<__half, __half, int8_t>(a, cs, ks);
  }
  if (a.dtype == B200MM_BF16) return launch_g<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16>(a, cs, ks);
  return launch_g<__half, __half, __half>(a, cs, ks);
}

}  // namespace b200mm
