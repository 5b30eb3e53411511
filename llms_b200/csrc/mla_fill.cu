// MLA side-band fill on the tensor cores (production shape: R = 256, D = 128,
// DR = 32, KV = 8, bf16 / fp16), for token ranges of a prefilled cache.
//
// The decode step needs, per cached token t and KV group g,
//   kscale[t, g] = rsqrt((|W_uk,g c_t|^2 + |kr_t,g|^2) / D + eps)
//   kz[t, g, :]  = rope_t(w_k[DN:] * kr_t,g)
// (the reference recomputes both for every token at every step,
// engine/mla.py:211-242).  The first term is a contraction
// [tokens x 256] . [256 x 768] whose output is only needed squared and summed
// per 96-column group, so it runs as a tcgen05 GEMM whose accumulators never
// leave the SM: tokens are the MMA's M side (128 per tile, one per TMEM lane),
// W_uk's rows its N side in chunks of 192 = two groups.
//
// Persistent, one CTA per SM over 128-token tiles of the flattened
// (batch row, token range) sequence; 11 warps:
//   warp 0      TMA: the tile's latent rows, one 4-D box [4 x 64 cols x 128
//               tokens] (64 KB, 128-byte swizzle), into a 2-slot ring, so the
//               next tile's rows stream in under this tile's MMAs;
//   warp 1      TMA: W_uk stages of two boxes [64 k x 192 rows] (48 KB, one
//               3-D load; all SMs read the same 393 KB from L2) into a
//               2-stage ring -- one stage per commit, since every
//               tcgen05.commit stalls the issuing thread;
//   warp 2      TMEM allocation; one thread issues tcgen05.mma (kind::f16,
//               M = 128, N = 192, K = 16) into two accumulator buffers of 192
//               columns, so chunk j + 1 accumulates while chunk j is read;
//   warps 3-10  two per TMEM lane quadrant: warp half h takes group 2n + h of
//               chunk n -- its 96 accumulator columns, squared and summed in
//               registers (the buffer goes back to the MMAs at once), then
//               the group's RoPE half from the token's own k_rope_pre row
//               (its squares, and kz).
// Every wait is bounded; a CTA whose wait expires stops issuing, drains its
// own copies, frees TMEM and writes NaN scales for its tokens.
#include "mla.cuh"
#include "tcgen05.cuh"

namespace b200mm {

namespace {

constexpr int FR = 256, FD = 128, FDR = 32, FKV = 8, FDN = FD - FDR;
constexpr int TM = 128;                          // tokens per tile (MMA M, TMEM lanes)
constexpr int CN = 192;                          // W_uk rows per chunk (MMA N): two groups
constexpr int NCHUNK = FKV * FDN / CN;           // 4
constexpr int KB = FR / 64;                      // 64-wide K boxes: 4
constexpr uint32_t A_BYTES = TM * FR * 2;        // 64 KB: one tile's latent rows
constexpr int WKB = 2;                           // K boxes per W stage (one TMA, one commit)
constexpr uint32_t W_BYTES = WKB * CN * 64 * 2;  // 48 KB: two W_uk boxes [64 k x 192 rows]
constexpr int A_SLOTS = 2, W_STAGES = 2;
constexpr uint32_t kTmemCols = 512;              // two accumulator buffers
constexpr uint32_t kBufCols = 256;               // buffer b at column 256 b (CN used)
constexpr int kThreads = 11 * 32;
constexpr int kEpi = 8 * 32;                     // epilogue threads
constexpr size_t kSmem = (size_t)A_SLOTS * A_BYTES + (size_t)W_STAGES * W_BYTES + 1024 + 256;
static_assert(FKV * FDN % CN == 0 && CN == 2 * FDN, "a chunk is exactly two groups");
static_assert(W_BYTES % 1024 == 0 && A_BYTES % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
static_assert(KB % WKB == 0, "a chunk's K boxes fill whole stages");
static_assert(kSmem + 1024 <= 232448, "shared memory (with the static arrays) fits one CTA");
static_assert(CN <= (int)kBufCols && 2 * kBufCols <= kTmemCols, "two accumulator buffers fit the allocation");

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const T lo = from_f<T>(a), hi = from_f<T>(b);
  return (uint32_t)(*reinterpret_cast<const uint16_t*>(&lo)) | ((uint32_t)(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
}

#ifdef FILL_TRACE
// Development trace (trace builds only): %globaltimer per (CTA < 4, tile < 8,
// event < 16), read back with b200mm_fill_trace.
__device__ unsigned long long g_fill_trace[4][8][16];
#define FTRACE(j, e)                                                                    \
  do {                                                                                  \
    if (blockIdx.x < 4 && (j) < 8) g_fill_trace[blockIdx.x][(j)][(e)] = global_ns();   \
  } while (0)
#else
#define FTRACE(j, e) \
  do {               \
  } while (0)
#endif

struct FillParams {
  int64_t t0, t1;
  int tiles_per_row, units;
  const void* kr; int64_t r_sb, r_st;
  void* kz; int64_t z_sb, z_st;
  float* kscale; int64_t s_sb, s_st;
  const float* k_norm_w; const float* inv_freq;
  float eps;
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    mla_fill_tc_kernel(const __grid_constant__ CUtensorMap mc, const __grid_constant__ CUtensorMap mw,
                       const FillParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  unsigned char* sa = sm;                                  // [A_SLOTS][A_BYTES]
  unsigned char* sw = sm + A_SLOTS * A_BYTES;              // [W_STAGES][W_BYTES]
  uint64_t* a_full = reinterpret_cast<uint64_t*>(sw + W_STAGES * W_BYTES);
  uint64_t* a_empty = a_full + A_SLOTS;
  uint64_t* w_full = a_empty + A_SLOTS;
  uint64_t* w_empty = w_full + W_STAGES;
  uint64_t* acc_full = w_empty + W_STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* failed = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* a_issued = const_cast<int*>(failed) + 1;
  int* a_used = a_issued + 1;
  int* w_issued = a_used + 1;
  int* w_used = w_issued + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mine = (int)blockIdx.x < p.units ? (p.units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < A_SLOTS; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < W_STAGES; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpi);  // every epilogue thread reads every chunk
    }
    mbar_init(mma_done, 1);
    *failed = 0;
    *a_issued = *a_used = *w_issued = *w_used = 0;
    mbar_init_fence();
    prefetch_map(&mc);
    prefetch_map(&mw);
  }
  // the RoPE half's k_norm weights and the RoPE frequencies, read by every
  // epilogue thread for every token: staged once
  __shared__ float s_kw[FDR], s_inv[FDR / 2];
  if (threadIdx.x < FDR) s_kw[threadIdx.x] = p.k_norm_w[FDN + threadIdx.x];
  if (threadIdx.x < FDR / 2) s_inv[threadIdx.x] = p.inv_freq[threadIdx.x];
  if (warp == 2) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_trigger();
  pdl_wait();  // the cache rows may come from the previous kernel

  if (warp == 0) {
    // ---------------- latent rows of each tile ----------------
    if (lane == 0) {
      int j = 0;
      for (; j < mine; ++j) {
        const int u = blockIdx.x + j * gridDim.x, b = u / p.tiles_per_row, i = u % p.tiles_per_row;
        const int s = j % A_SLOTS;
        if (j >= A_SLOTS && !mbar_wait(&a_empty[s], (uint32_t)(((j / A_SLOTS) - 1) & 1))) {
          *failed = 1;
          break;
        }
        if (*failed) break;
        mbar_expect_tx(&a_full[s], A_BYTES);
        FTRACE(j, 11);
        tma_load_4d(sa + s * A_BYTES, &mc, 0, (int)(p.t0 + (int64_t)i * TM), 0, b, &a_full[s]);
      }
      *a_issued = j;
    }
  } else if (warp == 1) {
    // ---------------- W_uk boxes: chunk n, K box kb, for every tile ----------------
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int j = 0; ok && j < mine; ++j)
        for (int n = 0; ok && n < NCHUNK; ++n)
          for (int kb = 0; kb < KB; kb += WKB, ++g) {
            const int s = g % W_STAGES;
            if (g >= W_STAGES && !mbar_wait(&w_empty[s], (uint32_t)(((g / W_STAGES) - 1) & 1))) ok = false;
            if (!ok || *failed) {
              ok = false;
              break;
            }
            mbar_expect_tx(&w_full[s], W_BYTES);
            tma_load_3d(sw + s * W_BYTES, &mw, 0, n * CN, kb, &w_full[s]);
          }
      if (!ok) *failed = 1;
      *w_issued = g;
    }
  } else if (warp == 2) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t ID = idesc_f16<T>(TM, CN);
      int g = 0, jc = 0, j = 0;
      bool ok = true;
      for (; ok && j < mine; ++j) {
        const int s = j % A_SLOTS;
        FTRACE(j, 0);
        if (!mbar_wait(&a_full[s], (uint32_t)((j / A_SLOTS) & 1)) || *failed) {
          ok = false;
          break;
        }
        tc_fence_after();
        FTRACE(j, 1);
        const uint32_t abase = smem_u32(sa + s * A_BYTES);
        for (int n = 0; ok && n < NCHUNK; ++n, ++jc) {
          const int buf = jc & 1;
          if (jc >= 2 && !mbar_wait(&acc_empty[buf], (uint32_t)(((jc >> 1) - 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + buf * kBufCols;
          for (int kb = 0; kb < KB; kb += WKB, ++g) {
            const int ws = g % W_STAGES;
            if (!mbar_wait(&w_full[ws], (uint32_t)((g / W_STAGES) & 1)) || *failed) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kw = 0; kw < WKB; ++kw) {
              const uint64_t ad = sdesc(abase + (kb + kw) * (TM * 128));
              const uint64_t bd = sdesc(smem_u32(sw + ws * W_BYTES + kw * (CN * 128)));
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) mma_f16(d, ad + 2 * kk, bd + 2 * kk, ID, (kb | kw | kk) != 0);
            }
            mma_commit(&w_empty[ws]);  // one commit per two K boxes: each commit stalls the issuer
          }
          if (ok) mma_commit(&acc_full[buf]);
          FTRACE(j, 2 + n);
        }
        if (ok) mma_commit(&a_empty[s]);  // the tile's rows may be overwritten once its MMAs complete
      }
      if (!ok) *failed = 1;
      *a_used = j;
      *w_used = g;
      mma_commit(mma_done);
    }
  } else {
    // ---------------- epilogue: warps 3..10 ----------------
    const int q = warp & 3, h = (warp - 3) >> 2;  // lane quadrant, group parity
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
    constexpr int half = FDR / 2;
    bool bad = false;
    int jc = 0;
    for (int j = 0; j < mine; ++j) {
      const int u = blockIdx.x + j * gridDim.x, b = u / p.tiles_per_row, i = u % p.tiles_per_row;
      const int64_t t = p.t0 + (int64_t)i * TM + 32 * q + lane;
      const bool valid = t < p.t1;
      const T* krow = static_cast<const T*>(p.kr) + (int64_t)b * p.r_sb + t * p.r_st + h * FDR;
      // k_rope_pre of this thread's groups, one chunk ahead of its use: the
      // loads are in flight while the accumulators are read and the previous
      // group is rotated
      uint4 kx[2][FDR / 8];
      auto load_kr = [&](uint4 (&dst)[FDR / 8], int n) {
#pragma unroll
        for (int c = 0; c < FDR / 8; ++c)
          dst[c] = valid ? *reinterpret_cast<const uint4*>(krow + 2 * n * FDR + 8 * c) : make_uint4(0, 0, 0, 0);
      };
      load_kr(kx[0], 0);
      float sn[half], cs[half];
      if (valid) {
#pragma unroll
        for (int ii = 0; ii < half; ++ii) sincosf((float)t * s_inv[ii], &sn[ii], &cs[ii]);
      }
      // chunk n holds groups 2n and 2n + 1: this warp takes group 2n + h --
      // its 96 accumulator columns first (so the buffer is handed back to the
      // MMAs at once), then the group's RoPE half from the token's own row
#pragma unroll
      for (int n = 0; n < NCHUNK; ++n, ++jc) {
        if (n + 1 < NCHUNK) load_kr(kx[(n + 1) & 1], n + 1);
        const int buf = jc & 1;
        float ssq = 0.f;
        if (!bad) {
          bad = !mbar_wait(&acc_full[buf], (uint32_t)((jc >> 1) & 1)) || *failed;
          tc_fence_after();
        }
        if (warp == 3 && lane == 0) FTRACE(j, 6 + n);
        if (!bad) {
#pragma unroll
          for (int c = 0; c < FDN; c += 32) {
            float v[32];
            tmem_ld32(tq + buf * kBufCols + h * FDN + c, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) ssq = fmaf(v[e], v[e], ssq);
          }
          tc_fence_before();
          mbar_arrive(&acc_empty[buf]);
        }
        if (!valid) continue;
        const int grp = 2 * n + h;
        float x[FDR];
#pragma unroll
        for (int c = 0; c < FDR / 8; ++c) Chunk<T>::unpack(kx[n & 1][c], x + 8 * c);
        float z[FDR];
#pragma unroll
        for (int jj = 0; jj < FDR; ++jj) {
          ssq = fmaf(x[jj], x[jj], ssq);
          const int ii = jj < half ? jj : jj - half;
          const float rot = jj < half ? -s_kw[jj + half] * x[jj + half] : s_kw[jj - half] * x[jj - half];
          z[jj] = s_kw[jj] * x[jj] * cs[ii] + rot * sn[ii];
        }
        T* dst = static_cast<T*>(p.kz) + (int64_t)b * p.z_sb + t * p.z_st + grp * FDR;
#pragma unroll
        for (int c = 0; c < FDR / 8; ++c) {
          uint4 o;
          o.x = pack2<T>(z[8 * c + 0], z[8 * c + 1]);
          o.y = pack2<T>(z[8 * c + 2], z[8 * c + 3]);
          o.z = pack2<T>(z[8 * c + 4], z[8 * c + 5]);
          o.w = pack2<T>(z[8 * c + 6], z[8 * c + 7]);
          *reinterpret_cast<uint4*>(dst + 8 * c) = o;
        }
        p.kscale[(int64_t)b * p.s_sb + t * p.s_st + grp] =
            bad ? __int_as_float(0x7fc00000) : rsqrtf(ssq / (float)FD + p.eps);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *failed) {
    // copies issued but never consumed still target this CTA's shared memory
    for (int j = *a_used; j < *a_issued; ++j) mbar_wait(&a_full[j % A_SLOTS], (uint32_t)((j / A_SLOTS) & 1));
    for (int g = *w_used; g < *w_issued; ++g) mbar_wait(&w_full[g % W_STAGES], (uint32_t)((g / W_STAGES) & 1));
  }
  if (threadIdx.x == 64) mbar_wait(mma_done, 0);
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

inline bool al16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

template <typename T>
int launch_t(const MlaAppendArgs& a) {
  const CUtensorMapDataType dt =
      a.s.dtype == B200MM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t B = (uint64_t)a.s.B, S = (uint64_t)a.t1;
  const uint64_t csb = B > 1 ? (uint64_t)a.c_sb * 2 : S * a.c_st * 2;
  // c as [batch][4 column blocks][token][64]: one box is a tile's 128 rows,
  // landing as four consecutive 128-byte-swizzled [128 x 64] K boxes; the
  // token extent is t1, so rows past the range arrive as zeros
  const uint64_t cd[4] = {64, S, 4, B};
  const uint64_t cs[3] = {(uint64_t)a.c_st * 2, 128, csb};
  const uint32_t box[4] = {64, (uint32_t)TM, 4, 1};
  CUtensorMap mc, mw;
  if (!make_map_4d(&mc, dt, a.c_kv, cd, cs, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_3d(&mw, dt, a.w_uk, 64, (uint64_t)FKV * FDN, KB, FR * 2, 128, 64, CN, WKB,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return B200MM_ERR_ALIGN;
  auto kern = mla_fill_tc_kernel<T>;
  static bool configured[64] = {false};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return B200MM_ERR_DEVICE;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) != cudaSuccess)
      return B200MM_ERR_LAUNCH;
    configured[dev] = true;
  }
  FillParams p{};
  p.t0 = a.t0;
  p.t1 = a.t1;
  const int64_t tpr = (a.t1 - a.t0 + TM - 1) / TM, units = tpr * (int64_t)a.s.B;
  if (units > 2147483647LL) return B200MM_ERR_SHAPE;
  p.tiles_per_row = (int)tpr;
  p.units = (int)units;
  p.kr = a.kr; p.r_sb = a.r_sb; p.r_st = a.r_st;
  p.kz = a.kz; p.z_sb = a.z_sb; p.z_st = a.z_st;
  p.kscale = a.kscale; p.s_sb = a.s_sb; p.s_st = a.s_st;
  p.k_norm_w = a.k_norm_w; p.inv_freq = a.inv_freq;
  p.eps = a.s.eps;
  const int sms = num_sms(dev);
  const int grid = (int)(units < sms ? units : sms);
  return launch_pdl(kern, dim3(grid), dim3(kThreads), kSmem, a.stream, mc, mw, p) == cudaSuccess
             ? B200MM_OK
             : B200MM_ERR_LAUNCH;
}

}  // namespace

bool mla_fill_tc_supported(const MlaAppendArgs& a) {
  const b200mm_mla_shape& s = a.s;
  if (s.R != FR || s.D != FD || s.DR != FDR || s.KV != FKV) return false;
  if (s.dtype != B200MM_BF16 && s.dtype != B200MM_F16) return false;
  if (a.t1 - a.t0 < kMlaFillTcMinTokens || a.t1 > (int64_t(1) << 30) || s.B < 1) return false;
  if (!al16(a.c_kv) || (a.c_st * 2) % 16 || (a.c_sb * 2) % 16 || a.c_st < FR) return false;
  if (!al16(a.w_uk) || !al16(a.kr) || (a.r_st * 2) % 16 || (a.r_sb * 2) % 16) return false;
  if (!al16(a.kz) || (a.z_st * 2) % 16 || (a.z_sb * 2) % 16) return false;
  return true;
}

#ifdef FILL_TRACE
extern "C" int b200mm_fill_trace(void* dst) {
  return cudaMemcpyFromSymbol(dst, g_fill_trace, sizeof(g_fill_trace)) == cudaSuccess ? 0 : 4;
}
#endif

int mla_fill_tc_launch(const MlaAppendArgs& a) {
  if (a.s.dtype == B200MM_BF16) return launch_t<__nv_bfloat16>(a);
  return launch_t<__half>(a);
}

}  // namespace b200mm
