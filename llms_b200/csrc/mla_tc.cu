// MLA latent decode, production shape (R=256, D=128, DR=32, H=32, KV=8;
// bf16 or fp16): the split kernel on 5th-generation tensor cores.
//
// One persistent CTA per SM walks its range of 64-token units (the plan in
// mla.cuh) with three roles:
//   warp 0      TMA producer: per unit, the latent rows c [64 tokens x 256]
//               and the RoPE'd-key side-band z [64 x 8*32] as four 64-column
//               boxes each (one 4-D TMA instruction per tensor: a TMA
//               instruction costs ~130 ns to issue whatever its size),
//               128-byte swizzled, plus the k-RMS side-band s [64 x 8]; a
//               ring of three stages guarded by full / empty mbarriers.
//   warps 1,6,7 one thread each issues tcgen05.mma (warp 1 also owns TMEM):
//                 scores  S[64 x 32] (M = 64 tokens, N = 32 heads):
//                           c-part  A = c box j, B = qt rows (K-major), 16
//                                   instructions of K = 16 over the 256 ranks;
//                           z-part  for each box j (groups 2j, 2j+1): A = z
//                                   box j, B = the RoPE queries of heads
//                                   8j..8j+7 placed in their group's 32
//                                   columns, N = 8, into those heads' columns
//                                   of a second score buffer.
//                 values  Acc[r][h] += sum_t c_t[r] P[h][t] for r in two
//                         halves of 128 (M = 128, N = 32, K = 64 tokens):
//                         A = the c boxes read MN-major (the latent index is
//                         the contiguous one), B = P [32 x 64] K-major; fp32
//                         accumulators stay in TMEM for the whole batch row.
//               Small MMAs are limited by one thread's issue rate, so warp 1
//               issues the c-part, warp 6 the z-part (into its own columns,
//               summed by the softmax) and warp 7 the values, each as soon as
//               its inputs are ready.
//   warps 2-5   softmax group.  An M = 64 accumulator puts token 16q + i in
//               lane i of TMEM quadrant q (lanes 16-31 unused), so warp q's
//               lanes 0-15 read their token's 32 scores and lanes 16-31 take
//               heads 16-31 of the same tokens by shuffle: each thread owns
//               one token x 16 heads.  Scale by s_t,g * scale * log2(e),
//               per-head maxima and sums by transposing butterflies plus a
//               4-warp exchange, P = 2^(S - m) in the storage dtype; the
//               running maximum moves lazily (only when a unit's maximum
//               exceeds it by more than 8, so P <= 256) and then the group
//               rescales the accumulators in TMEM.  At the end of a batch row
//               the group writes the (acc, max, sum) partial.
//
// Every mbarrier wait is bounded (%globaltimer); on expiry the kernel sets
// the workspace error flag, stops issuing, waits (bounded) for its own copies
// and MMAs in flight, frees TMEM and returns; the combine kernel then writes
// NaN outputs.
#include "mla.cuh"
#include "tcgen05.cuh"

namespace b200mm {

namespace {

constexpr int FR = 256, FD = 128, FDR = 32, FH = 32, FKV = 8;
constexpr int TT = kMlaUnit;  // 64 tokens per unit
constexpr int kThr = 256;  // warps: 0 TMA, 1 scores c-part, 2-5 softmax, 6 scores z-part, 7 values
constexpr int NST = 3;                             // stages in the ring
constexpr uint32_t kBox = TT * 128;                // [64 rows x 128 B]: 8 KB
constexpr uint32_t kZOff = 4 * kBox;               // z boxes after the four c boxes
constexpr uint32_t kSOff = 8 * kBox;               // s side-band
constexpr uint32_t kStage = kSOff + TT * FKV * 4;  // 66 KB per unit
constexpr uint32_t kQtBytes = 4 * FH * 128;        // qt: four K-chunks of [32 rows x 128 B]
constexpr uint32_t kQrBytes = 4 * 8 * 128;         // qr: four [8 rows x 128 B] blocks
constexpr uint32_t kPBytes = FH * 128;             // P: [32 heads x 64 tokens]
constexpr uint32_t kTmemCols = 256;  // c-part scores 2 x 32 columns, z-part 2 x 32, accumulators 64
constexpr uint32_t kZCol = 64, kAccCol = 128;
constexpr float kLazy = 8.f;  // log2 units: P <= 256
constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
static_assert(kStage % 1024 == 0, "stages must keep the 1024-byte swizzle-atom alignment");

#ifdef MLA_TC_TRACE
// Development trace: per CTA, per unit (first 16), %globaltimer at eight
// points, written past the end of the planned workspace.
#define TRACE(which, j)                                                                              \
  do {                                                                                               \
    if ((j) < 16)                                                                                    \
      reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(a.ws) +                      \
                                            w.total)[(cta * 8 + (which)) * 16 + (j)] = global_ns(); \
  } while (0)
#else
#define TRACE(which, j) \
  do {                  \
  } while (0)
#endif

struct __align__(1024) TcSmem {
  unsigned char stage[NST][kStage];
  unsigned char qt[kQtBytes];
  unsigned char qr[kQrBytes];
  unsigned char p[kPBytes];
  float red_max[4][FH];
  float red_sum[4][FH];
  float m[FH];  // running (lazy) maximum per head, log2 units
  float l[FH];  // running sum per head
  float alpha[FH];
  int need;
  int failed;
  int issued, consumed[2];
  uint32_t tmem;
  unsigned long long full[NST], empty[NST], s_full[2], s_empty[2], p_full, pv_done, q_ready, mma_done[3];
};

__device__ __forceinline__ void nbar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// Barrier over `n` threads that also returns the AND of `v` across them.
__device__ __forceinline__ bool nbar_and(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// Transposing butterfly over each half-warp: v[i] is this lane's value for
// head hb + i; returns the reduction over the 16 lanes of this half of head
// hb + (lane % 16).  15 shuffles.
template <bool MAX>
__device__ __forceinline__ float xreduce16(const float* in, int lane) {
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = in[i];
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
    const bool up = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float keep = up ? v[i + w] : v[i];
      const float send = up ? v[i] : v[i + w];
      const float got = __shfl_xor_sync(0xffffffffu, send, w);
      v[i] = MAX ? fmaxf(keep, got) : keep + got;
    }
  }
  return v[0];
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 128-byte swizzled position of 16-byte chunk `c` of row `row`.
__device__ __forceinline__ uint32_t sw_chunk(int row, int c) { return (uint32_t)(row * 128 + ((c ^ (row & 7)) << 4)); }

template <typename T>
__global__ void __launch_bounds__(kThr, 1)
    mla_tc_split_kernel(const MlaDecodeArgs a, MlaWorkspace w, const __grid_constant__ CUtensorMap map_c,
                        const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_s) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  TcSmem& S = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* failed = &S.failed;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  MLA_SPAN(1, 0);
  const int cta = blockIdx.x;
  float* ws = static_cast<float*>(a.ws);
  int* err = reinterpret_cast<int*>(static_cast<unsigned char*>(a.ws) + w.off_err);

  const int64_t u_begin = mla_range_begin(w, cta), u_end = mla_range_begin(w, cta + 1);
  const int n = (int)(u_end - u_begin);
  auto row_of = [&](int j) { return (int)((u_begin + j) / w.ntiles); };
  auto t0_of = [&](int j) { return (int)((u_begin + j - (int64_t)row_of(j) * w.ntiles) * TT); };

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&S.s_full[s], 2);     // c-part and z-part issuers
      mbar_init(&S.s_empty[s], 128);  // the softmax group has read the buffer
    }
    mbar_init(&S.p_full, 128);
    mbar_init(&S.pv_done, 1);
    mbar_init(&S.q_ready, 128);
    for (int s = 0; s < 3; ++s) mbar_init(&S.mma_done[s], 1);
    S.failed = 0;
    S.issued = 0;
    S.consumed[0] = S.consumed[1] = 0;
    mbar_init_fence();
    prefetch_map(&map_c);
    prefetch_map(&map_z);
    prefetch_map(&map_s);
  }
  if (warp == 1) tmem_alloc(&S.tmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;

  // one unit's cache rows: the four c boxes, the four z boxes (one 4-D TMA
  // instruction each) and the k-RMS side-band
  auto issue = [&](int j) {
    const int st = j % NST, b = row_of(j), t0 = t0_of(j);
    unsigned char* sb = S.stage[st];
    TRACE(0, j);
    mbar_expect_tx(&S.full[st], kStage);
    tma_load_4d(sb, &map_c, 0, t0, 0, b, &S.full[st]);
    tma_load_4d(sb + kZOff, &map_z, 0, t0, 0, b, &S.full[st]);
    tma_load_3d(sb + kSOff, &map_s, 0, t0, b, &S.full[st]);
  };
  // The absorb kernel releases this one only after its own predecessor (the
  // cache append) finished, so the cache may be fetched before the wait; the
  // absorbed queries (workspace) are read after it.
  const int pre = n < NST ? n : NST;
  if (tid == 0)
    for (int j = 0; j < pre; ++j) issue(j);
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int j = pre;
      for (; j < n; ++j) {
        const int st = j % NST;
        if (j >= NST && !mbar_wait(&S.empty[st], (uint32_t)(((j - NST) / NST) & 1))) {
          *failed = 1;
          break;
        }
        if (*failed) break;
        issue(j);
      }
      S.issued = j;
    }
  } else if (warp == 1 || warp == 6) {
    // ---------------- score issuers: warp 1 c-part, warp 6 z-part ----------------
    // Small MMAs are bound by how fast one thread can issue them, so the two
    // halves of the scores come from two threads, each into its own columns.
    if (lane == 0 && n > 0) {
      const bool zpart = warp == 6;
      constexpr uint32_t IDC = idesc_f16<T>(64, 32);  // c-part: 32 heads
      constexpr uint32_t IDZ = idesc_f16<T>(64, 8);   // z-part: the 8 heads of one z box
      const uint32_t qt_addr = smem_u32(S.qt), qr_addr = smem_u32(S.qr);
      int rr = 0;  // q_ready phases consumed (batch rows)
      bool ok = mbar_wait(&S.q_ready, 0) && !*failed;
      rr = 1;
      int j = 0;
      for (; ok && j < n; ++j) {
        if (j > 0 && row_of(j) != row_of(j - 1)) {  // a new batch row: wait for its queries
          if (!(ok = mbar_wait(&S.q_ready, (uint32_t)(rr & 1)) && !*failed)) break;
          ++rr;
        }
        const int st = j % NST, sb = j & 1;
        if (!(ok = mbar_wait(&S.full[st], (uint32_t)((j / NST) & 1)) && !*failed)) break;
        if (j >= 2 && !(ok = mbar_wait(&S.s_empty[sb], (uint32_t)(((j - 2) >> 1) & 1)) && !*failed)) break;
        TRACE(zpart ? 6 : 1, j);
        tc_fence_after();
        const uint32_t base = smem_u32(S.stage[st]);
        if (!zpart) {
          const uint32_t d = tmem + 32 * sb;
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int k16 = 0; k16 < 4; ++k16)
              mma_f16(d, sdesc(base + c * kBox) + 2 * k16, sdesc(qt_addr + c * (FH * 128)) + 2 * k16, IDC,
                      (c | k16) != 0);
        } else {
          const uint32_t d = tmem + kZCol + 32 * sb;
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int k16 = 0; k16 < 4; ++k16)
              mma_f16(d + 8 * c, sdesc(base + kZOff + c * kBox) + 2 * k16, sdesc(qr_addr + c * 1024) + 2 * k16,
                      IDZ, k16 != 0);
        }
        mma_commit(&S.s_full[sb]);
        TRACE(zpart ? 7 : 5, j);
      }
      if (!ok) *failed = 1;
      S.consumed[zpart ? 1 : 0] = j;
      mma_commit(&S.mma_done[zpart ? 1 : 0]);
      mbar_wait(&S.mma_done[zpart ? 1 : 0], 0);  // no MMA may still write TMEM when it is freed
    }
  } else if (warp == 7) {
    // ---------------- values issuer ----------------
    if (lane == 0 && n > 0) {
      constexpr uint32_t IDP = idesc_f16<T>(128, 32, /*a_mn=*/true);
      const uint32_t paddr = smem_u32(S.p);
      bool ok = true;
      for (int k = 0; k < n; ++k) {
        if (!(ok = mbar_wait(&S.p_full, (uint32_t)(k & 1)) && !*failed)) break;
        TRACE(4, k);
        tc_fence_after();
        const bool first = k == 0 || row_of(k) != row_of(k - 1);
        const uint32_t base = smem_u32(S.stage[k % NST]);
#pragma unroll
        for (int mh = 0; mh < 2; ++mh)
#pragma unroll
          for (int k16 = 0; k16 < 4; ++k16)
            mma_f16(tmem + kAccCol + 32 * mh, sdesc_mn(base + 2 * mh * kBox + k16 * 2048, kBox),
                    sdesc(paddr) + 2 * k16, IDP, !(first && k16 == 0));
        // the scores of unit k finished before its softmax began, so the stage is free with these
        mma_commit(&S.empty[k % NST]);
        mma_commit(&S.pv_done);
      }
      if (!ok) *failed = 1;
      mma_commit(&S.mma_done[2]);
      mbar_wait(&S.mma_done[2], 0);
    }
  } else {
    // ---------------- softmax group: warps 2-5 ----------------
    const int q = warp & 3;                // TMEM lane quadrant
    const int tok = 16 * q + (lane & 15);  // token within the unit
    const int hb = lane & 16;              // this thread's heads: hb .. hb+15
    const int gt = tid - 64;               // 0..127 inside the group
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
    auto load_q = [&](int b) {  // queries of batch row b, storage dtype, K-major swizzled
      const float* qt = ws + w.off_qt / 4 + (int64_t)b * FH * FR;
      const float* qr = ws + w.off_qr / 4 + (int64_t)b * FH * FDR;
      constexpr int QI = FH * 32 / 128;  // qt: 32 rows x 32 chunks of 8, QI per thread, all loads first
      float4 v[QI][2];
#pragma unroll
      for (int u = 0; u < QI; ++u) {
        const int i = gt + 128 * u, row = i >> 5, k0 = 8 * (i & 31);
        v[u][0] = *reinterpret_cast<const float4*>(qt + row * FR + k0);
        v[u][1] = *reinterpret_cast<const float4*>(qt + row * FR + k0 + 4);
      }
#pragma unroll
      for (int u = 0; u < QI; ++u) {
        const int i = gt + 128 * u, row = i >> 5, c8 = i & 31;
        uint4 o;
        o.x = pack2<T>(v[u][0].x, v[u][0].y);
        o.y = pack2<T>(v[u][0].z, v[u][0].w);
        o.z = pack2<T>(v[u][1].x, v[u][1].y);
        o.w = pack2<T>(v[u][1].z, v[u][1].w);
        *reinterpret_cast<uint4*>(S.qt + (c8 >> 3) * (FH * 128) + sw_chunk(row, c8 & 7)) = o;
      }
      {  // qr block j, row i = head 8j+i; nonzero in its group's 32 columns of box j
        const int blk = gt >> 5, i = (gt >> 2) & 7, c2 = gt & 3;  // 4 blocks x 8 rows x 4 pairs of chunks
        const int h = 8 * blk + i, half = i >> 2;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * c2 + cc;  // chunk 0..7 of the 64 columns
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int col = 8 * c + e;
            f[e] = (col >> 5) == half ? qr[h * FDR + (col & 31)] : 0.f;
          }
          uint4 o;
          o.x = pack2<T>(f[0], f[1]);
          o.y = pack2<T>(f[2], f[3]);
          o.z = pack2<T>(f[4], f[5]);
          o.w = pack2<T>(f[6], f[7]);
          *reinterpret_cast<uint4*>(S.qr + blk * 1024 + sw_chunk(i, c)) = o;
        }
      }
      fence_proxy_async();  // generic-proxy writes, read by the tensor core
    };
    auto flush = [&](int b) {  // accumulators + statistics -> partial slot cta + b
      const int64_t slot = (int64_t)cta + b;
      float* pacc = ws + w.off_pacc / 4 + slot * FH * FR;
#pragma unroll 1
      for (int mh = 0; mh < 2; ++mh) {
        float v[32];
        tmem_ld32(tq + kAccCol + 32 * mh, v);
        const int r = 128 * mh + 32 * q + lane;
#pragma unroll
        for (int h = 0; h < FH; ++h) pacc[(int64_t)h * FR + r] = v[h];
      }
      if (q == 0) {
        float* pml = ws + w.off_pml / 4 + slot * FH * 2;
        pml[2 * lane] = S.m[lane] * kLn2;  // the merge works in natural-log units
        pml[2 * lane + 1] = S.l[lane];
      }
    };

    bool ok = true;
    if (n > 0) {
      if (q == 0) {
        S.m[lane] = -INFINITY;
        S.l[lane] = 0.f;
      }
      load_q(row_of(0));
      mbar_arrive(&S.q_ready);
    }
    const float qscale = a.scale * kLog2e;
    for (int k = 0; k < n; ++k) {
      const int st = k % NST, sb = k & 1;
      const bool first = k == 0 || row_of(k) != row_of(k - 1);
      const int nv = (int)imin64(TT, a.L - t0_of(k));
      ok = nbar_and(1, 128, mbar_wait(&S.s_full[sb], (uint32_t)((k >> 1) & 1)) && !*failed);
      if (!ok) break;
      if (gt == 0) TRACE(2, k);
      tc_fence_after();
      float u[16];
      {
        float v[32], vz[32];
        tmem_ld32(tq + 32 * sb, v);  // lanes 0-15: token tok, heads 0-31
        tmem_ld32(tq + kZCol + 32 * sb, vz);
        tc_fence_before();
        mbar_arrive(&S.s_empty[sb]);  // both halves are in registers
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += vz[i];
        const float4 s4 = *(reinterpret_cast<const float4*>(S.stage[st] + kSOff) + 2 * tok + (hb >> 4));
        const float sg[4] = {s4.x * qscale, s4.y * qscale, s4.z * qscale, s4.w * qscale};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float hi = __shfl_sync(0xffffffffu, v[16 + i], lane & 15);
          const float x = (hb ? hi : v[i]) * sg[i >> 2];
          u[i] = tok < nv ? x : -INFINITY;
        }
      }
      {
        const float mx = xreduce16<true>(u, lane);
        S.red_max[q][hb + (lane & 15)] = mx;
      }
      nbar(1, 128);
      if (q == 0) {  // lane = head: lazy running maximum (log2 units)
        const float mu = fmaxf(fmaxf(S.red_max[0][lane], S.red_max[1][lane]),
                               fmaxf(S.red_max[2][lane], S.red_max[3][lane]));  // finite: a unit has a token
        const float mo = S.m[lane];
        const float mn = (mo == -INFINITY || mu > mo + kLazy) ? fmaxf(mu, mo) : mo;
        const bool any = __any_sync(0xffffffffu, mn != mo);
        S.alpha[lane] = mo == -INFINITY ? 0.f : ex2(mo - mn);
        S.m[lane] = mn;
        if (lane == 0) S.need = any ? 1 : 0;
      }
      nbar(1, 128);
      const bool rescale = S.need && !first;
      float p[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) p[i] = ex2(u[i] - S.m[hb + i]);
      {
        const float sm = xreduce16<false>(p, lane);
        S.red_sum[q][hb + (lane & 15)] = sm;
      }
      // values of unit k-1 are done: P and the accumulators are free
      if (k > 0) {
        ok = nbar_and(1, 128, mbar_wait(&S.pv_done, (uint32_t)((k - 1) & 1)) && !*failed);
        if (!ok) break;
        tc_fence_after();
      }
      if (rescale) {
#pragma unroll 1
        for (int mh = 0; mh < 2; ++mh) {
          float acc[32];
          tmem_ld32(tq + kAccCol + 32 * mh, acc);
#pragma unroll
          for (int h = 0; h < FH; ++h) acc[h] *= S.alpha[h];
          tmem_st32(tq + kAccCol + 32 * mh, acc);
        }
      }
      {
        T* pp = reinterpret_cast<T*>(S.p);
#pragma unroll
        for (int i = 0; i < 16; ++i) pp[(sw_chunk(hb + i, tok >> 3) >> 1) + (tok & 7)] = from_f<T>(p[i]);
        fence_proxy_async();
      }
      tc_fence_before();
      if (gt == 0) TRACE(3, k);
      mbar_arrive(&S.p_full);
      nbar(1, 128);
      if (q == 0)
        S.l[lane] = S.l[lane] * S.alpha[lane] +
                    ((S.red_sum[0][lane] + S.red_sum[1][lane]) + (S.red_sum[2][lane] + S.red_sum[3][lane]));
      const bool last = k + 1 == n || row_of(k + 1) != row_of(k);
      if (last) {
        if (k + 1 < n) {  // the scores of unit k are done with the queries: load the next row's
          load_q(row_of(k + 1));
          mbar_arrive(&S.q_ready);
        }
        ok = nbar_and(1, 128, mbar_wait(&S.pv_done, (uint32_t)(k & 1)) && !*failed);
        if (!ok) break;
        tc_fence_after();
        flush(row_of(k));
        if (q == 0) {
          S.m[lane] = -INFINITY;
          S.l[lane] = 0.f;
        }
        tc_fence_before();
        nbar(1, 128);
      }
    }
    if (!ok) *failed = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *failed) {
    atomicExch(err, 1);
    // copies issued but never consumed still target this CTA's shared memory
    const int c0 = S.consumed[0] < S.consumed[1] ? S.consumed[0] : S.consumed[1];
    for (int j = c0; j < S.issued; ++j) mbar_wait(&S.full[j % NST], (uint32_t)((j / NST) & 1));
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  MLA_SPAN(1, 1);
}

}  // namespace

size_t mla_tc_smem_bytes() { return sizeof(TcSmem) + 1024; }

int mla_tc_split_launch(const MlaDecodeArgs& a, const MlaWorkspace& w, const MlaMaps& m) {
  const size_t smem = mla_tc_smem_bytes();
  static bool configured[2][64] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return B200MM_ERR_DEVICE;
  const int which = a.s.dtype == B200MM_BF16 ? 0 : 1;
  auto kern = which == 0 ? mla_tc_split_kernel<__nv_bfloat16> : mla_tc_split_kernel<__half>;
  if (!configured[which][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return B200MM_ERR_LAUNCH;
    configured[which][dev] = true;
  }
  return launch_pdl(kern, dim3(w.G), dim3(kThr), smem, a.stream, a, w, m.c, m.kz, m.ks) == cudaSuccess
             ? B200MM_OK
             : B200MM_ERR_LAUNCH;
}

}  // namespace b200mm
