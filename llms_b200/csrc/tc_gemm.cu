// Large-M projection kernel on 5th-generation tensor cores (tcgen05).
//
//   Y[M, N] = X[M, K] . W[N, K]^T            (fused QKV: W = [Wq; Wk; Wv])
//   Y[M, N] = silu(X Wg^T) * (X Wu^T)        (fused gate-up-SiLU)
//
// Persistent: one CTA per SM walks 128 x BN output tiles (BN x 2 for
// gate-up; m-tiles vary fastest), 6 warps:
//   warp 0      TMA producer: X box [64 k x 128 rows], W box(es) [64 k x BN
//               rows], 128-byte swizzle, into a STAGES-deep ring guarded by
//               full/empty mbarriers, continuous across the CTA's tiles;
//   warp 1      allocates TMEM, one thread issues tcgen05.mma (kind::f16,
//               M = 128, N = BN, K = 16 per instruction, fp32 accumulator in
//               TMEM) and frees each stage with tcgen05.commit; tile j
//               accumulates into buffer j & 1, so the epilogue of tile j
//               overlaps the main loop of tile j + 1;
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp reads its
//               32-lane quadrant), SiLU * up in registers for gate-up, one
//               rounding to the output dtype, 16-byte stores, then the buffer
//               is handed back to the issuer.
// Every mbarrier wait is bounded; a CTA whose wait expires stops issuing,
// drains its own copies in flight, frees TMEM and writes NaN over its tiles.
#include <type_traits>

#include "dense.cuh"
#include "tcgen05.cuh"

namespace b200mm {

namespace {

constexpr int BM = 128;  // tile rows (X rows) = MMA M = TMEM lanes
constexpr int BK = 64;   // K per stage: 128 bytes of 16-bit elements (one swizzle span)
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;  // two accumulator buffers (one CTA per SM)

template <bool GATE, int BN>
struct Cfg {
  static constexpr int NB = GATE ? 2 : 1;                // W tiles per stage
  static constexpr uint32_t A_BYTES = BM * BK * 2;       // 16 KB
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + NB * B_BYTES;
  static constexpr int STAGES = (200 * 1024 / STAGE_BYTES) > 8 ? 8 : (200 * 1024 / STAGE_BYTES);
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(NB * BN <= (int)kTmemCols, "accumulators exceed the TMEM allocation");
  static_assert(BN % 16 == 0 && BN >= 32 && NB * BN <= 256, "MMA N = NB * BN must be a multiple of 16 in [32, 256]");
  static_assert(B_BYTES % 1024 == 0, "W boxes must keep the 1024-byte swizzle-atom alignment");
};

struct TcParams {
  int M, N, K;
  void* y;
  int64_t ldy;
};

// kind::f16 instruction descriptor for this kernel's M = BM tiles.
template <typename T, int N>
constexpr uint32_t idesc() {
  return idesc_f16<T>(BM, N);
}

template <int WC>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, float* v) {
  if constexpr (WC == 32) tmem_ld32(taddr, v);
  else tmem_ld16(taddr, v);
}

template <typename T> __device__ __forceinline__ uint32_t pack_out(float a, float b);
template <> __device__ __forceinline__ uint32_t pack_out<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack_out<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T, bool GATE, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mw0,
                   const __grid_constant__ CUtensorMap mw1, const TcParams p) {
  using C = Cfg<GATE, BN>;
  constexpr uint32_t ACC = C::NB * BN;  // TMEM columns of one tile's accumulators
  constexpr uint32_t BUF = kTmemCols / 2;  // buffer b starts at column BUF * b (256-aligned)
  static_assert(ACC <= BUF, "two accumulator buffers must fit the TMEM allocation");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;  // [2]: a tile's accumulators are complete
  uint64_t* acc_empty = acc_full + 2;      // [2]: the epilogue has read them
  uint64_t* mma_done = acc_empty + 2;      // every MMA of this CTA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* issued = const_cast<int*>(failed) + 1;
  int* consumed = issued + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Persistent: CTA c takes tiles c, c + G, ...; m-tiles vary fastest, so the
  // tiles in flight at once cover all of X against a narrow band of W (each
  // weight row leaves HBM once, X stays in L2).
  const int mt = (p.M + BM - 1) / BM, ntl = (p.N + BN - 1) / BN, tiles = mt * ntl;
  const int mine = blockIdx.x < tiles ? (tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(mma_done, 1);
    *failed = 0;
    *issued = 0;
    *consumed = 0;
    mbar_init_fence();
    prefetch_map(&mx);
    prefetch_map(&mw0);
    if (GATE) prefetch_map(&mw1);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_trigger();
  pdl_wait();  // X may be the output of the previous kernel

  if (warp == 0) {
    // ---------------- TMA producer: one ring across all of this CTA's tiles ----------------
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int j = 0; ok && j < mine; ++j) {
        const int t = blockIdx.x + j * gridDim.x, tm = t % mt, tn = t / mt;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % C::STAGES, it = g / C::STAGES;
          if (g >= C::STAGES && !mbar_wait(&empty[s], (uint32_t)((it - 1) & 1))) ok = false;
          if (!ok || *failed) {
            ok = false;
            break;
          }
          unsigned char* st = sm + s * C::STAGE_BYTES;
          mbar_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d(st, &mx, kb * BK, tm * BM, &full[s]);
          tma_load_2d(st + C::A_BYTES, &mw0, kb * BK, tn * BN, &full[s]);
          if (GATE) tma_load_2d(st + C::A_BYTES + C::B_BYTES, &mw1, kb * BK, tn * BN, &full[s]);
        }
      }
      if (!ok) *failed = 1;
      *issued = g;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: tile j accumulates into buffer j & 1 ----------------
    if (lane == 0) {
      // gate-up: the Wg and Wu boxes are adjacent in shared memory, so one
      // N = 2*BN instruction reads A once and fills [gate | up] accumulators
      constexpr uint32_t ID = idesc<T, GATE ? 2 * BN : BN>();
      int g = 0;
      bool ok = true;
      for (int j = 0; ok && j < mine; ++j) {
        const int b = j & 1;
        // the epilogue of tile j - 2 must have read this buffer
        if (j >= 2 && !mbar_wait(&acc_empty[b], (uint32_t)(((j >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + b * BUF;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % C::STAGES, it = g / C::STAGES;
          if (!mbar_wait(&full[s], (uint32_t)(it & 1)) || *failed) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(sm + s * C::STAGE_BYTES);
          const uint64_t a = sdesc(st), bd = sdesc(st + C::A_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // +32 bytes of K per instruction inside the 128-byte swizzle span
            mma_f16(d, a + 2 * kk, bd + 2 * kk, ID, (kb | kk) != 0);
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);  // fires once the tile's MMAs have completed
      }
      if (!ok) *failed = 1;
      *consumed = g;
      // let every MMA issued above finish before TMEM can be freed (its own
      // barrier: one more arrival on acc_full could run ahead of the epilogue)
      mma_commit(mma_done);
    }
  } else {
    // ---------------- epilogue: warps 2..5 -> TMEM lane quadrant warp % 4 ----------------
    const int q = warp & 3;
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
    bool bad = false;
    for (int j = 0; j < mine; ++j) {
      const int t = blockIdx.x + j * gridDim.x, tm = t % mt, tn = t / mt;
      const int b = j & 1;
      if (!bad) {
        bad = !mbar_wait(&acc_full[b], (uint32_t)((j >> 1) & 1)) || *failed;
        tc_fence_after();
      }
      const int row = tm * BM + 32 * q + lane;
      T* yrow = static_cast<T*>(p.y) + (int64_t)row * p.ldy;
#pragma unroll 1
      // one block of WC accumulator columns (32, or a 16-column tail when
      // BN is an odd multiple of 16): TMEM -> registers -> 16-byte stores
      auto cols = [&](int c, auto wc) {
        constexpr int WC = decltype(wc)::value;
        float v[WC];
        if (!bad) {
          tmem_ldn<WC>(tq + b * BUF + c, v);
          if (GATE) {
            float u[WC];
            tmem_ldn<WC>(tq + b * BUF + BN + c, u);
#pragma unroll
            for (int i = 0; i < WC; ++i) v[i] = silu_mul(v[i], u[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < WC; ++i) v[i] = __int_as_float(0x7fc00000);
        }
        if (row < p.M) {
          const int n0 = tn * BN + c;
          if (n0 + WC <= p.N) {
#pragma unroll
            for (int jj = 0; jj < WC / 8; ++jj) {
              uint4 o;
              o.x = pack_out<T>(v[8 * jj + 0], v[8 * jj + 1]);
              o.y = pack_out<T>(v[8 * jj + 2], v[8 * jj + 3]);
              o.z = pack_out<T>(v[8 * jj + 4], v[8 * jj + 5]);
              o.w = pack_out<T>(v[8 * jj + 6], v[8 * jj + 7]);
              *reinterpret_cast<uint4*>(yrow + n0 + 8 * jj) = o;
            }
          } else {
#pragma unroll
            for (int i = 0; i < WC; ++i)
              if (n0 + i < p.N) yrow[n0 + i] = from_f<T>(v[i]);
          }
        }
      };
#pragma unroll 1
      for (int c = 0; c + 32 <= BN; c += 32) cols(c, std::integral_constant<int, 32>{});
      if constexpr (BN % 32 != 0) cols(BN - 16, std::integral_constant<int, 16>{});
      if (!bad) {
        tc_fence_before();
        mbar_arrive(&acc_empty[b]);  // buffer b may take tile j + 2
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *failed) {
    // copies issued but never consumed still target this CTA's shared memory
    for (int g = *consumed; g < *issued; ++g) mbar_wait(&full[g % C::STAGES], (uint32_t)((g / C::STAGES) & 1));
  }
  if (threadIdx.x == 32) mbar_wait(mma_done, 0);
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

template <typename T>
constexpr CUtensorMapDataType map_dtype() {
  return sizeof(T) == 2 && ab_format<T>() == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

template <typename T, bool GATE, int BN>
int launch_bn(const DenseArgs& a) {
  using C = Cfg<GATE, BN>;
  CUtensorMap mx, mw0, mw1;
  const CUtensorMapDataType dt = map_dtype<T>();
  if (!make_map_2d(&mx, dt, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.ldx * 2, BK, BM,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&mw0, dt, a.w0, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.ldw0 * 2, BK, BN,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return B200MM_ERR_ALIGN;
  if (GATE) {
    if (!make_map_2d(&mw1, dt, a.w1, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.ldw1 * 2, BK, BN,
                     CU_TENSOR_MAP_SWIZZLE_128B))
      return B200MM_ERR_ALIGN;
  } else {
    mw1 = mw0;
  }
  auto kern = tc_gemm_kernel<T, GATE, BN>;
  static bool configured[64] = {false};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return B200MM_ERR_DEVICE;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) != cudaSuccess)
      return B200MM_ERR_LAUNCH;
    configured[dev] = true;
  }
  TcParams p{a.M, a.N, a.K, a.y, a.ldy};
  const long tiles = (long)((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
  if (tiles > 2147483647L) return B200MM_ERR_SHAPE;
  const int sms = num_sms(dev);
  dim3 grid((unsigned)(tiles < sms ? tiles : sms));  // persistent: one CTA per SM
  return launch_pdl(kern, grid, dim3(kThreads), C::SMEM, a.stream, mx, mw0, mw1, p) == cudaSuccess
             ? B200MM_OK
             : B200MM_ERR_LAUNCH;
}

// N tile: the one with the least streaming per SM.  A CTA's tile reads
// BM x K of X and (2 x) BN x K of W, and the persistent grid takes
// ceil(tiles / SMs) rounds, so cost(BN) = rounds x (BM + NB * BN) -- e.g. at
// M = 128 gate-up, 76 tiles of BN = 128 in one round beat 152 tiles of
// BN = 64 in two.
template <typename T>
int launch_t(const DenseArgs& a) {
  const long sms = num_sms(current_device());
  const long mt = (a.M + BM - 1) / BM;
  auto cost = [&](int bn, int nb) {
    const long tiles = mt * ((a.N + bn - 1) / bn);
    return ((tiles + sms - 1) / sms) * (long)(BM + nb * bn);
  };
  if (a.gate) {
    const long c128 = cost(128, 2), c64 = cost(64, 2);
    return c128 <= c64 ? launch_bn<T, true, 128>(a) : launch_bn<T, true, 64>(a);
  }
  const long c256 = cost(256, 1), c128 = cost(128, 1), c64 = cost(64, 1);
  if (c256 <= c128 && c256 <= c64) return launch_bn<T, false, 256>(a);
  if (c128 <= c64) return launch_bn<T, false, 128>(a);
  return launch_bn<T, false, 64>(a);
}

}  // namespace

bool tc_supported(const DenseArgs& a) {
  if (a.w8 || (a.dtype != B200MM_BF16 && a.dtype != B200MM_F16)) return false;
  if (a.M < 65) return false;
  if (!al16(a.x) || !al16(a.w0) || !al16(a.y) || (a.gate && !al16(a.w1))) return false;
  if ((a.ldx * 2) % 16 || (a.ldw0 * 2) % 16 || (a.ldy * 2) % 16 || (a.gate && (a.ldw1 * 2) % 16)) return false;
  if ((a.K * 2) % 16) return false;
  return true;
}

int tc_launch(const DenseArgs& a) {
  if (a.dtype == B200MM_BF16) return launch_t<__nv_bfloat16>(a);
  return launch_t<__half>(a);
}

}  // namespace b200mm
