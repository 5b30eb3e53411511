// MLA latent decode, production shape (R=256, D=128, DR=32, H=32, KV=8;
// bf16 or fp16): the split kernel on tensor cores.
//
// One persistent CTA per SM walks its range of 64-token units (see the plan
// in mla.cuh).  Per unit:
//   1. TMA tensor loads (3-D maps over [batch, token, channel], token extent
//      L so rows past the context arrive as zeros) bring c [64 x 256] and
//      k_rope_pre [64 x 8*32] as four 64-column boxes each, 128-byte swizzled,
//      and the k-RMS side-band [64 x 8]; completion on an mbarrier; two
//      stages, so the next unit streams while this one computes;
//   2. z = rope_t(w_k[DN:] * kr) per (token, group) on CUDA cores, written
//      over k_rope_pre in place;
//   3. scores S[64 x 32] = C . Qt^T (K = 256) + Z . Qr^T (per group, K = 64)
//      on mma.sync m16n8k16 (fp32 accumulate), then * s_t,g * scale;
//   4. online softmax per head (running max / sum in shared memory);
//   5. acc[32 x 256] = acc * alpha + P . C on mma.sync (registers, 32 fp32
//      per thread), P in the storage dtype.
// A CTA writes one (acc, max, sum) partial per batch row it touched.
//
// Every mbarrier wait is bounded (%globaltimer); on expiry the kernel sets
// the workspace error flag, waits (bounded) for its own copies in flight and
// returns; the combine kernel then writes NaN outputs.
#include "mla.cuh"

#ifndef MLA_SKIP
#define MLA_SKIP 0  // development knob: bitmask of phases to skip when timing (0 in every build)
#endif

namespace b200mm {

namespace {

constexpr int FR = 256, FD = 128, FDR = 32, FDN = 96, FH = 32, FKV = 8;
constexpr int TT = kMlaUnit;      // 64 tokens per unit
constexpr int NT = 256;           // threads
constexpr int CP = FR + 8;        // padded row pitch (elements) of c / kr / z / qt: 528 bytes
constexpr int PP = TT + 8;        // P row pitch: 144 bytes
constexpr int RP = 64 + 8;        // rope-query row pitch
constexpr int SCP = FH + 1;       // score row pitch (fp32)

constexpr uint32_t kTileBytes = TT * FR * 2;                 // one [64 x 256] 16-bit tile: 32 KB
constexpr uint32_t kUnitBytes = 2 * kTileBytes + TT * FKV * 4;  // c + kr + side-band per unit

// c and kr tiles are four [64 rows x 128 B] boxes in the TMA 128-byte swizzle
// (see sw128_off); the struct is placed at a 1024-byte aligned address.
template <typename T>
struct __align__(1024) FastSmem {
  unsigned char c[2][kTileBytes];
  unsigned char kr[2][kTileBytes];
  float s[2][TT][FKV];
  T qt[FH][CP];
  T qrb[FH][RP];
  T p[FH][PP];
  float sc[TT][SCP];
  float cs[TT][16];
  float sn[TT][16];
  float m[FH], l[FH], alpha[FH];
  unsigned long long bar[2];
};

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(p)));
}

template <typename T> struct Mma;
template <> struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct Mma<__half> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t v);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<__half2*>(&v));
}

struct Unit {
  int b;
  int64_t t0;
  int nv;
};

template <typename T>
__global__ void __launch_bounds__(NT, 1)
    mla_fast_split_kernel(const MlaDecodeArgs a, MlaWorkspace w, const __grid_constant__ CUtensorMap map_c,
                          const __grid_constant__ CUtensorMap map_kr, const __grid_constant__ CUtensorMap map_s) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  FastSmem<T>& S = *reinterpret_cast<FastSmem<T>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cta = blockIdx.x;
  float* ws = static_cast<float*>(a.ws);
  int* err = reinterpret_cast<int*>(static_cast<unsigned char*>(a.ws) + w.off_err);

  const int64_t u_begin = mla_range_begin(w, cta), u_end = mla_range_begin(w, cta + 1);
  auto unit_of = [&](int64_t u) {
    Unit r;
    r.b = (int)(u / w.ntiles);
    r.t0 = (u - (int64_t)r.b * w.ntiles) * TT;
    r.nv = (int)imin64(TT, a.L - r.t0);
    return r;
  };
  // Issue the loads of unit u into stage st (one thread).
  auto issue = [&](int64_t u, int st) {
    const Unit un = unit_of(u);
    mbar_expect_tx(&S.bar[st], kUnitBytes);
    for (int j = 0; j < 4; ++j) {
      tma_load_3d(S.c[st] + j * TT * 128, &map_c, 64 * j, (int)un.t0, un.b, &S.bar[st]);
      tma_load_3d(S.kr[st] + j * TT * 128, &map_kr, 64 * j, (int)un.t0, un.b, &S.bar[st]);
    }
    tma_load_3d(&S.s[st][0][0], &map_s, 0, (int)un.t0, un.b, &S.bar[st]);
  };

  if (tid == 0) {
    mbar_init(&S.bar[0], 1);
    mbar_init(&S.bar[1], 1);
    mbar_init_fence();
    prefetch_map(&map_c);
    prefetch_map(&map_kr);
    prefetch_map(&map_s);
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // the cache, side-band and absorbed query come from earlier kernels

  if (tid == 0) {
    issue(u_begin, 0);
    if (u_begin + 1 < u_end) issue(u_begin + 1, 1);
  }

  // per-thread constants: the rope weights / frequencies this thread uses
  const int zi2 = tid & 7;  // pair index: dims i = 2*zi2, 2*zi2+1 (and +16)
  float wlo[2], whi[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    wlo[e] = a.k_norm_w[FDN + 2 * zi2 + e];
    whi[e] = a.k_norm_w[FDN + 16 + 2 * zi2 + e];
  }
  const float my_freq = a.inv_freq[tid & 15];

  float acc[2][4][4];
  int cur_b = -1;
  bool bad = false;
  int64_t k = 0;  // local unit counter (stage = k & 1, parity = (k >> 1) & 1)

  auto flush = [&](int b) {
    const int64_t slot = (int64_t)cta + b;
    float* pacc = ws + w.off_pacc / 4 + slot * FH * FR;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int h = 16 * mt + (lane >> 2) + 8 * hf;
          const int r = 32 * warp + 8 * nt + 2 * (lane & 3);
          *reinterpret_cast<float2*>(pacc + (int64_t)h * FR + r) =
              make_float2(acc[mt][nt][2 * hf], acc[mt][nt][2 * hf + 1]);
        }
    if (tid < FH) {
      float* pml = ws + w.off_pml / 4 + slot * FH * 2;
      pml[2 * tid] = S.m[tid];
      pml[2 * tid + 1] = S.l[tid];
    }
  };

  for (int64_t u = u_begin; u < u_end; ++u, ++k) {
    const Unit un = unit_of(u);
    const int st = (int)(k & 1);
    if (un.b != cur_b) {
      if (cur_b >= 0) flush(cur_b);
      __syncthreads();
      // absorbed query of row b -> shared (storage dtype), rope query -> block layout
      const float* qt = ws + w.off_qt / 4 + (int64_t)un.b * FH * FR;
      for (int i = tid; i < FH * FR / 2; i += NT) {
        const int h = (2 * i) / FR, r = (2 * i) % FR;
        const float2 v = *reinterpret_cast<const float2*>(qt + (int64_t)h * FR + r);
        *reinterpret_cast<uint32_t*>(&S.qt[h][r]) = pack2<T>(v.x, v.y);
      }
      const float* qr = ws + w.off_qr / 4 + (int64_t)un.b * FH * FDR;
      for (int i = tid; i < FH * 64; i += NT) {
        const int h = i / 64, kk = i % 64;
        const int lg = (h & 7) >> 2;  // this head's group within its 8-head n-tile
        const float v = (kk / 32 == lg) ? qr[h * FDR + (kk & 31)] : 0.f;
        S.qrb[h][kk] = from_f<T>(v);
      }
      if (tid < FH) { S.m[tid] = -INFINITY; S.l[tid] = 0.f; }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
      cur_b = un.b;
    }
    // cos / sin of this unit's positions (independent of the copies)
    for (int i = tid; i < TT * 16; i += NT) {
      const int t = i >> 4;
      float sv, cv;
      if (MLA_SKIP & 1) { sv = 0.5f; cv = 0.5f; } else
      sincosf((float)(un.t0 + t) * my_freq, &sv, &cv);
      S.cs[t][i & 15] = cv;
      S.sn[t][i & 15] = sv;
    }
    if (!mbar_wait(&S.bar[st], (uint32_t)((k >> 1) & 1))) {
      bad = true;
    }
    if (__syncthreads_or(bad)) {
      bad = true;
      break;
    }
    __syncthreads();

    // ---- z[t][g*32 + j] = rope_t(w_r * kr[t][g])[j], in place over kr ----
    for (int it = tid; it < ((MLA_SKIP & 2) ? 0 : TT * FKV * 8); it += NT) {
      const int tg = it >> 3, t = tg >> 3, g = tg & 7;
      const int i = 2 * zi2;
      unsigned char* base = S.kr[st];
      uint32_t* plo = reinterpret_cast<uint32_t*>(base + sw128_off(t, g * FDR + i, TT));
      uint32_t* phi = reinterpret_cast<uint32_t*>(base + sw128_off(t, g * FDR + 16 + i, TT));
      const float2 lo = unpack2<T>(*plo);
      const float2 hi = unpack2<T>(*phi);
      const float c0 = S.cs[t][i], c1 = S.cs[t][i + 1], s0 = S.sn[t][i], s1 = S.sn[t][i + 1];
      const float l0 = wlo[0] * lo.x, l1 = wlo[1] * lo.y, h0 = whi[0] * hi.x, h1 = whi[1] * hi.y;
      *plo = pack2<T>(l0 * c0 - h0 * s0, l1 * c1 - h1 * s1);
      *phi = pack2<T>(h0 * c0 + l0 * s0, h1 * c1 + l1 * s1);
    }
    __syncthreads();

    // ---- scores: warp -> token m-tile (warp>>1), head n-tiles 2*(warp&1) + {0,1} ----
    {
      const int mt = warp >> 1, nt0 = (warp & 1) * 2;
      float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const int arow = 16 * mt + (lane & 15), acol = 8 * (lane >> 4);
      const int bmat = lane >> 3, brow = 8 * nt0 + (bmat >> 1) * 8 + (lane & 7), bcol = (bmat & 1) * 8;
#pragma unroll 4
      for (int ks = 0; ks < ((MLA_SKIP & 4) ? 0 : FR / 16); ++ks) {
        uint32_t af[4], b0, b1, b2, b3;
        ldsm_x4(S.c[st] + sw128_off(arow, 16 * ks + acol, TT), af[0], af[1], af[2], af[3]);
        ldsm_x4(&S.qt[brow][16 * ks + bcol], b0, b1, b2, b3);
        Mma<T>::run(sacc[0], af, b0, b1);
        Mma<T>::run(sacc[1], af, b2, b3);
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int np = nt0 + q;  // covers groups 2np, 2np+1 -> z columns [64np, 64np+64)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          uint32_t af[4], b0, b1;
          ldsm_x4(S.kr[st] + sw128_off(arow, 64 * np + 16 * ks + acol, TT), af[0], af[1], af[2], af[3]);
          ldsm_x2(&S.qrb[8 * np + (lane & 7)][16 * ks + ((lane >> 3) & 1) * 8], b0, b1);
          Mma<T>::run(sacc[q], af, b0, b1);
        }
      }
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * mt + (lane >> 2) + 8 * (e >> 1);
          const int h = 8 * (nt0 + q) + 2 * (lane & 3) + (e & 1);
          const float v = sacc[q][e] * S.s[st][t][h >> 2] * a.scale;
          S.sc[t][h] = t < un.nv ? v : -INFINITY;
        }
    }
    __syncthreads();

    // ---- online softmax: 8 threads per head, 8 tokens each ----
    {
      const int h = tid >> 3, sub = tid & 7;
      float v[8], mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = S.sc[sub * 8 + j][h];
        mx = fmaxf(mx, v[j]);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      const float m_old = S.m[h];
      const float m_new = fmaxf(m_old, mx);  // finite: every unit has >= 1 valid token
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float p0 = __expf(v[j] - m_new), p1 = __expf(v[j + 1] - m_new);
        sum += p0 + p1;
        *reinterpret_cast<uint32_t*>(&S.p[h][sub * 8 + j]) = pack2<T>(p0, p1);
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      __syncwarp();
      if (sub == 0) {
        const float al = __expf(m_old - m_new);
        S.alpha[h] = al;
        S.l[h] = S.l[h] * al + sum;
        S.m[h] = m_new;
      }
    }
    __syncthreads();

    // ---- acc = acc * alpha + P . C ; warp -> latent cols [32*warp, +32) ----
    {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const float a0 = S.alpha[16 * mt + (lane >> 2)], a1 = S.alpha[16 * mt + 8 + (lane >> 2)];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          acc[mt][nt][0] *= a0; acc[mt][nt][1] *= a0;
          acc[mt][nt][2] *= a1; acc[mt][nt][3] *= a1;
        }
      }
      const int prow = lane & 15, pcol = 8 * (lane >> 4);
      const int bk = ((lane >> 3) & 1) * 8 + (lane & 7), bn = (lane >> 4) * 8;
#pragma unroll
      for (int ks = 0; ks < ((MLA_SKIP & 8) ? 0 : TT / 16); ++ks) {
        uint32_t pa[2][4];
        ldsm_x4(&S.p[prow][16 * ks + pcol], pa[0][0], pa[0][1], pa[0][2], pa[0][3]);
        ldsm_x4(&S.p[16 + prow][16 * ks + pcol], pa[1][0], pa[1][1], pa[1][2], pa[1][3]);
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(S.c[st] + sw128_off(16 * ks + bk, 32 * warp + 16 * pp + bn, TT), b0, b1, b2, b3);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            Mma<T>::run(acc[mt][2 * pp], pa[mt], b0, b1);
            Mma<T>::run(acc[mt][2 * pp + 1], pa[mt], b2, b3);
          }
        }
      }
    }
    fence_proxy_async();  // order this thread's generic accesses of stage st before the async refill
    __syncthreads();      // every read of stage st is done
    if (tid == 0 && u + 2 < u_end) issue(u + 2, st);
  }

  if (bad) {
    if (tid == 0) atomicExch(err, 1);
    // let copies still in flight land before the CTA's shared memory goes away
    const int64_t issued = (u_end - u_begin) < 2 ? (u_end - u_begin) : 2;
    for (int64_t j = k; j < k + issued && j < (u_end - u_begin); ++j) mbar_wait(&S.bar[j & 1], (uint32_t)((j >> 1) & 1));
    return;
  }
  if (cur_b >= 0) flush(cur_b);
}

template <typename T>
int launch_fast(const MlaDecodeArgs& a, const MlaWorkspace& w, const MlaMaps& m) {
  auto kern = mla_fast_split_kernel<T>;
  const size_t smem = sizeof(FastSmem<T>) + 1024;  // + slack for the 1024-byte alignment
  static bool configured[64] = {false};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return B200MM_ERR_DEVICE;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return B200MM_ERR_LAUNCH;
    configured[dev] = true;
  }
  return launch_pdl(kern, dim3(w.G), dim3(NT), smem, a.stream, a, w, m.c, m.kr, m.ks) == cudaSuccess
             ? B200MM_OK
             : B200MM_ERR_LAUNCH;
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

int mla_fast_ctas() { return num_sms(current_device()); }

bool mla_fast_supported(const MlaDecodeArgs& a) {
  const b200mm_mla_shape& s = a.s;
  if (s.R != FR || s.D != FD || s.DR != FDR || s.H != FH || s.KV != FKV) return false;
  if (s.dtype != B200MM_BF16 && s.dtype != B200MM_F16) return false;
  if (a.L > (int64_t(1) << 30) || s.B < 1) return false;
  // TMA: 16-byte aligned bases and strides, rows no shorter than their content
  if (!al16(a.c_kv) || (a.c_st * 2) % 16 || (a.c_sb * 2) % 16 || a.c_st < FR) return false;
  if (!al16(a.kr) || (a.r_st * 2) % 16 || (a.r_sb * 2) % 16 || a.r_st < FKV * FDR) return false;
  if (!al16(a.kscale) || (a.s_st * 4) % 16 || (a.s_sb * 4) % 16 || a.s_st < FKV) return false;
  return true;
}

bool mla_fast_maps(const MlaDecodeArgs& a, MlaMaps* m) {
  const CUtensorMapDataType dt =
      a.s.dtype == B200MM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t L = (uint64_t)a.L, B = (uint64_t)a.s.B;
  // a single batch row may come with any batch stride; give the map a valid one
  const uint64_t csb = B > 1 ? (uint64_t)a.c_sb * 2 : L * a.c_st * 2;
  const uint64_t rsb = B > 1 ? (uint64_t)a.r_sb * 2 : L * a.r_st * 2;
  const uint64_t ssb = B > 1 ? (uint64_t)a.s_sb * 4 : L * a.s_st * 4;
  return make_map_3d(&m->c, dt, a.c_kv, FR, L, B, (uint64_t)a.c_st * 2, csb, 64, TT, 1, CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_map_3d(&m->kr, dt, a.kr, FKV * FDR, L, B, (uint64_t)a.r_st * 2, rsb, 64, TT, 1,
                     CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_map_3d(&m->ks, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.kscale, FKV, L, B, (uint64_t)a.s_st * 4, ssb, FKV,
                     TT, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int mla_fast_split_launch(const MlaDecodeArgs& a, const MlaWorkspace& w, const MlaMaps& maps) {
  if (a.s.dtype == B200MM_BF16) return launch_fast<__nv_bfloat16>(a, w, maps);
  return launch_fast<__half>(a, w, maps);
}

}  // namespace b200mm
