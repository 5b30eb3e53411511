// MLA latent decode, production shape (R=256, D=128, DR=32, H=32, KV=8;
// bf16 or fp16): the split kernel on tensor cores.
//
// One persistent CTA per SM walks its range of 64-token units (see the plan
// in mla.cuh).  Per unit:
//   1. TMA tensor loads (3-D maps over [batch, token, channel], token extent
//      L so rows past the context arrive as zeros) bring c [64 x 256] and the
//      RoPE'd key side-band z [64 x 8*32] as four 64-column boxes each,
//      128-byte swizzled, and the k-RMS side-band s [64 x 8]; completion on an
//      mbarrier; two stages, so the next unit streams while this one computes;
//   2. scores S[64 x 32] = C . Qt^T (K = 256) + Z . Qr^T (per 8-head n-tile,
//      the 64 z columns of its two groups) on mma.sync m16n8k16, fp32
//      accumulate, two independent accumulator chains per tile;
//   3. S * s_t,g * scale stays in the MMA fragments; per-head max across the
//      four token warps through shared memory; P = exp(S - m) in the storage
//      dtype; per-head sums;
//   4. acc[32 x 256] = acc * alpha + P . C on mma.sync (registers, 32 fp32 per
//      thread).  The running max is double-buffered by unit parity, so a unit
//      needs three CTA barriers.
// A CTA writes one (acc, max, sum) partial per batch row it touched.
//
// Every mbarrier wait is bounded (%globaltimer); on expiry the kernel sets
// the workspace error flag, waits (bounded) for its own copies in flight and
// returns; the combine kernel then writes NaN outputs.
#include "mla.cuh"

namespace b200mm {

namespace {

constexpr int FR = 256, FD = 128, FDR = 32, FH = 32, FKV = 8;
constexpr int TT = kMlaUnit;      // 64 tokens per unit
constexpr int NT = 256;           // threads
constexpr int CP = FR + 8;        // padded row pitch (elements) of qt: 528 bytes
constexpr int PP = TT + 8;        // P row pitch: 144 bytes
constexpr int RP = 64 + 8;        // rope-query row pitch

constexpr uint32_t kTileBytes = TT * FR * 2;                     // one [64 x 256] 16-bit tile: 32 KB
constexpr uint32_t kUnitBytes = 2 * kTileBytes + TT * FKV * 4;    // c + z + s per unit

// c and z tiles are four [64 rows x 128 B] boxes in the TMA 128-byte swizzle
// (see sw128_off); the struct is placed at a 1024-byte aligned address.
template <typename T>
struct __align__(1024) FastSmem {
  unsigned char c[2][kTileBytes];
  unsigned char z[2][kTileBytes];
  float s[2][TT][FKV];
  T qt[FH][CP];
  T qrb[FH][RP];
  T p[FH][PP];
  float red_max[4][FH];  // per token m-tile, per head
  float red_sum[4][FH];
  float m[2][FH];        // running max, double-buffered by unit parity
  float l[FH];
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

struct Unit {
  int b;
  int64_t t0;
  int nv;
};

__device__ __forceinline__ float max4(const float (*rm)[FH], int h) {
  return fmaxf(fmaxf(rm[0][h], rm[1][h]), fmaxf(rm[2][h], rm[3][h]));
}

template <typename T>
__global__ void __launch_bounds__(NT, 1)
    mla_fast_split_kernel(const MlaDecodeArgs a, MlaWorkspace w, const __grid_constant__ CUtensorMap map_c,
                          const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_s) {
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
      tma_load_3d(S.z[st] + j * TT * 128, &map_z, 64 * j, (int)un.t0, un.b, &S.bar[st]);
    }
    tma_load_3d(&S.s[st][0][0], &map_s, 0, (int)un.t0, un.b, &S.bar[st]);
  };

  if (tid == 0) {
    mbar_init(&S.bar[0], 1);
    mbar_init(&S.bar[1], 1);
    mbar_init_fence();
    prefetch_map(&map_c);
    prefetch_map(&map_z);
    prefetch_map(&map_s);
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // the cache, side-bands and absorbed query come from earlier kernels
  if (tid == 0) {
    issue(u_begin, 0);
    if (u_begin + 1 < u_end) issue(u_begin + 1, 1);
  }

  // scores: warp -> token m-tile mt_s (16 tokens), head n-tiles nt0, nt0 + 1
  const int mt_s = warp >> 1, nt0 = (warp & 1) * 2;
  const int r0 = 16 * mt_s + (lane >> 2);  // this lane's fragment rows r0, r0 + 8
  const int cq = 2 * (lane & 3);           // fragment column pair

  float acc[2][4][4];  // P.C: heads 16*mt + lane/4 (+8), latent 32*warp + 8*nt + cq (+1)
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
          const int r = 32 * warp + 8 * nt + cq;
          *reinterpret_cast<float2*>(pacc + (int64_t)h * FR + r) =
              make_float2(acc[mt][nt][2 * hf], acc[mt][nt][2 * hf + 1]);
        }
    if (tid < FH) {
      float* pml = ws + w.off_pml / 4 + slot * FH * 2;
      pml[2 * tid] = S.m[k & 1][tid];
      pml[2 * tid + 1] = S.l[tid];
    }
  };

  for (int64_t u = u_begin; u < u_end; ++u, ++k) {
    const Unit un = unit_of(u);
    const int st = (int)(k & 1), mb = (int)(k & 1);  // stage; running-max buffer read this unit
    if (un.b != cur_b) {
      if (cur_b >= 0) flush(cur_b);
      __syncthreads();
      // absorbed query of row b -> shared (storage dtype); rope query -> per-n-tile block layout
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
      if (tid < FH) { S.m[mb][tid] = -INFINITY; S.l[tid] = 0.f; }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.f;
      cur_b = un.b;
      __syncthreads();
    }

    if (!mbar_wait(&S.bar[st], (uint32_t)((k >> 1) & 1))) bad = true;
    if (__syncthreads_or(bad)) {
      bad = true;
      break;
    }

    // ---- scores S[t][h] = c_t . qt_h + z_t,g . qr_h ----
    float sacc[2][4], sacc2[2][4];
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int e = 0; e < 4; ++e) sacc[q][e] = sacc2[q][e] = 0.f;
    {
      const unsigned char* cbase = S.c[st];
      const int arow = 16 * mt_s + (lane & 15), acol = 8 * (lane >> 4);
      const int bmat = lane >> 3, brow = 8 * nt0 + (bmat >> 1) * 8 + (lane & 7), bcol = (bmat & 1) * 8;
#pragma unroll 4
      for (int ks = 0; ks < FR / 16; ks += 2) {
        uint32_t af[4], ag[4], b0, b1, b2, b3, d0, d1, d2, d3;
        ldsm_x4(cbase + sw128_off(arow, 16 * ks + acol, TT), af[0], af[1], af[2], af[3]);
        ldsm_x4(&S.qt[brow][16 * ks + bcol], b0, b1, b2, b3);
        ldsm_x4(cbase + sw128_off(arow, 16 * ks + 16 + acol, TT), ag[0], ag[1], ag[2], ag[3]);
        ldsm_x4(&S.qt[brow][16 * ks + 16 + bcol], d0, d1, d2, d3);
        Mma<T>::run(sacc[0], af, b0, b1);
        Mma<T>::run(sacc[1], af, b2, b3);
        Mma<T>::run(sacc2[0], ag, d0, d1);
        Mma<T>::run(sacc2[1], ag, d2, d3);
      }
      // rope part: n-tile np uses the 64 z columns of its groups 2np, 2np+1
      const unsigned char* zbase = S.z[st];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int np = nt0 + q;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          uint32_t af[4], b0, b1;
          ldsm_x4(zbase + sw128_off(arow, 64 * np + 16 * ks + acol, TT), af[0], af[1], af[2], af[3]);
          ldsm_x2(&S.qrb[8 * np + (lane & 7)][16 * ks + ((lane >> 3) & 1) * 8], b0, b1);
          Mma<T>::run((ks & 1) ? sacc2[q] : sacc[q], af, b0, b1);
        }
      }
    }
    // scale by s_t,g * scale, mask tokens past the context, per-head max over this warp's 16 rows
#pragma unroll
    for (int q = 0; q < 2; ++q) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = r0 + 8 * (e >> 1);
        const int h = 8 * (nt0 + q) + cq + (e & 1);
        const float v = (sacc[q][e] + sacc2[q][e]) * S.s[st][t][h >> 2] * a.scale;
        sacc[q][e] = t < un.nv ? v : -INFINITY;
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float m = fmaxf(sacc[q][c], sacc[q][2 + c]);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        if (lane < 4) S.red_max[mt_s][8 * (nt0 + q) + cq + c] = m;
      }
    }
    __syncthreads();
    // ---- softmax numerators: p = exp(s - m_new), P[h][t] in the storage dtype ----
#pragma unroll
    for (int q = 0; q < 2; ++q) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int h = 8 * (nt0 + q) + cq + c;
        const float m_new = fmaxf(max4(S.red_max, h), S.m[mb][h]);  // finite: every unit has a valid token
        const float p0 = __expf(sacc[q][c] - m_new), p1 = __expf(sacc[q][2 + c] - m_new);
        S.p[h][r0] = from_f<T>(p0);
        S.p[h][r0 + 8] = from_f<T>(p1);
        float sum = p0 + p1;
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        sum += __shfl_xor_sync(0xffffffffu, sum, 8);
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        if (lane < 4) S.red_sum[mt_s][h] = sum;
      }
    }
    __syncthreads();
    // ---- acc = acc * alpha + P . C ; warp -> latent cols [32*warp, +32) ----
    {
      if (tid < FH) {  // running statistics; the new max goes to the other buffer
        const float m_old = S.m[mb][tid];
        const float m_new = fmaxf(max4(S.red_max, tid), m_old);
        const float tsum = (S.red_sum[0][tid] + S.red_sum[1][tid]) + (S.red_sum[2][tid] + S.red_sum[3][tid]);
        S.l[tid] = S.l[tid] * __expf(m_old - m_new) + tsum;
        S.m[mb ^ 1][tid] = m_new;
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int h = 16 * mt + (lane >> 2) + 8 * hf;
          const float m_old = S.m[mb][h];
          const float al = __expf(m_old - fmaxf(max4(S.red_max, h), m_old));
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            acc[mt][nt][2 * hf] *= al;
            acc[mt][nt][2 * hf + 1] *= al;
          }
        }
      }
      const int prow = lane & 15, pcol = 8 * (lane >> 4);
      const int bk = ((lane >> 3) & 1) * 8 + (lane & 7), bn = (lane >> 4) * 8;
      const unsigned char* cbase = S.c[st];
#pragma unroll
      for (int ks = 0; ks < TT / 16; ++ks) {
        uint32_t pa[2][4];
        ldsm_x4(&S.p[prow][16 * ks + pcol], pa[0][0], pa[0][1], pa[0][2], pa[0][3]);
        ldsm_x4(&S.p[16 + prow][16 * ks + pcol], pa[1][0], pa[1][1], pa[1][2], pa[1][3]);
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(cbase + sw128_off(16 * ks + bk, 32 * warp + 16 * pp + bn, TT), b0, b1, b2, b3);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            Mma<T>::run(acc[mt][2 * pp], pa[mt], b0, b1);
            Mma<T>::run(acc[mt][2 * pp + 1], pa[mt], b2, b3);
          }
        }
      }
    }
    fence_proxy_async();  // order this thread's shared-memory accesses before the async refill
    __syncthreads();      // every read of stage st, P and the reduction buffers is done
    if (tid == 0 && u + 2 < u_end) issue(u + 2, st);
  }

  if (bad) {
    if (tid == 0) atomicExch(err, 1);
    // let copies still in flight land before the CTA's shared memory goes away
    const int64_t n = u_end - u_begin;
    for (int64_t j = k; j < k + 2 && j < n; ++j) mbar_wait(&S.bar[j & 1], (uint32_t)((j >> 1) & 1));
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
  return launch_pdl(kern, dim3(w.G), dim3(NT), smem, a.stream, a, w, m.c, m.kz, m.ks) == cudaSuccess
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
  if (!al16(a.kz) || (a.z_st * 2) % 16 || (a.z_sb * 2) % 16 || a.z_st < FKV * FDR) return false;
  if (!al16(a.kscale) || (a.s_st * 4) % 16 || (a.s_sb * 4) % 16 || a.s_st < FKV) return false;
  return true;
}

bool mla_fast_maps(const MlaDecodeArgs& a, MlaMaps* m) {
  const CUtensorMapDataType dt =
      a.s.dtype == B200MM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t L = (uint64_t)a.L, B = (uint64_t)a.s.B;
  // a single batch row may come with any batch stride; give the map a valid one
  const uint64_t csb = B > 1 ? (uint64_t)a.c_sb * 2 : L * a.c_st * 2;
  const uint64_t zsb = B > 1 ? (uint64_t)a.z_sb * 2 : L * a.z_st * 2;
  const uint64_t ssb = B > 1 ? (uint64_t)a.s_sb * 4 : L * a.s_st * 4;
  return make_map_3d(&m->c, dt, a.c_kv, FR, L, B, (uint64_t)a.c_st * 2, csb, 64, TT, 1, CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_map_3d(&m->kz, dt, a.kz, FKV * FDR, L, B, (uint64_t)a.z_st * 2, zsb, 64, TT, 1,
                     CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_map_3d(&m->ks, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.kscale, FKV, L, B, (uint64_t)a.s_st * 4, ssb, FKV,
                     TT, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int mla_fast_split_launch(const MlaDecodeArgs& a, const MlaWorkspace& w, const MlaMaps& maps) {
  if (a.s.dtype == B200MM_BF16) return launch_fast<__nv_bfloat16>(a, w, maps);
  return launch_fast<__half>(a, w, maps);
}

}  // namespace b200mm
