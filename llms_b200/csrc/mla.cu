// MLA latent-KV decode with absorbed up-projections (any shape).
//
// The reference decode step (engine/mla.py:195-264) rebuilds K and V for all
// L cached tokens every step: V = W_uv c_t, K = k_norm([W_uk c_t ; kr_t]),
// partial RoPE on the last DR dims, GQA expansion, SDPA.  Here the step reads
// each cached token once, in latent form:
//
//   s_t,g     = rsqrt(mean_d k_t,g[d]^2 + eps)        (side-band, written at append)
//   z_t,g     = rope_t(w_k[DN:] * kr_t,g)              (side-band, written at append)
//   qt_h      = W_uk,g^T (w_k[:DN] * q_h[:DN])         (absorbed query, per step)
//   qr_h      = rope_{L-1}(q_h[DN:])
//   score_t,h = scale * s_t,g * (qt_h . c_t + qr_h . z_t,g)
//   out_h     = W_uv,g (sum_t softmax(score)_t,h c_t)
//
// which equals the reference because k_norm multiplies the raw head by the
// scalar s_t,g and then by w_k elementwise, and RoPE is linear.  The context
// is split into S chunks per batch row (flash-decoding); each split writes a
// partial (max, sum, sum p c) and a combine kernel merges the splits and
// applies W_uv once per head.
#include "mla.cuh"

namespace b200mm {

namespace {

constexpr int kThreads = 256;
constexpr int kTileT = 16;  // tokens per tile in the generic split kernel

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i) { return to_f<T>(p[i]); }

// --- per-token side-bands (at append) ----------------------------------------
// grid: (ceil((t1-t0)/8), B); block 256.  Each CTA handles 8 tokens of one
// batch row; warps walk the KV*DN rows of W_uk, lanes split the rank.
template <typename T>
__global__ void __launch_bounds__(kThreads) mla_append_kernel(const MlaAppendArgs a) {
  extern __shared__ float sm[];
  const int R = a.s.R, KV = a.s.KV, D = a.s.D, DR = a.s.DR, DN = D - DR, half = DR / 2;
  constexpr int TT = 8;
  float* cs = sm;                 // [TT][R]
  float* ssq = sm + TT * R;       // [TT][KV]
  const int b = blockIdx.y;
  const int64_t tb = a.t0 + (int64_t)blockIdx.x * TT;
  const int nt = (int)imin64(TT, a.t1 - tb);
  const T* c = static_cast<const T*>(a.c_kv) + (int64_t)b * a.c_sb;
  const T* kr = static_cast<const T*>(a.kr);
  const T* wuk = static_cast<const T*>(a.w_uk);

  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < TT * R; i += blockDim.x) {
    const int t = i / R, r = i % R;
    cs[i] = t < nt ? ldf(c, (tb + t) * a.c_st + r) : 0.f;
  }
  for (int i = threadIdx.x; i < TT * KV; i += blockDim.x) ssq[i] = 0.f;
  __syncthreads();
  // rope half: its sum of squares, and z = rope_t(w_k[DN:] * kr)
  for (int i = threadIdx.x; i < TT * KV * DR; i += blockDim.x) {
    const int t = i / (KV * DR), rem = i % (KV * DR), g = rem / DR, j = rem % DR;
    if (t >= nt) continue;
    const T* p = kr + (int64_t)b * a.r_sb + (tb + t) * a.r_st + (int64_t)g * DR;
    const float x = ldf(p, j);
    atomicAdd(&ssq[t * KV + g], x * x);
    const int ii = j < half ? j : j - half;
    float sn, cn;
    sincosf((float)(tb + t) * a.inv_freq[ii], &sn, &cn);
    const float rot = j < half ? -a.k_norm_w[DN + j + half] * ldf(p, j + half)
                               : a.k_norm_w[DN + j - half] * ldf(p, j - half);
    T* zp = static_cast<T*>(a.kz) + (int64_t)b * a.z_sb + (tb + t) * a.z_st + (int64_t)g * DR;
    zp[j] = from_f<T>(a.k_norm_w[DN + j] * x * cn + rot * sn);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int row = warp; row < KV * DN; row += nw) {
    const int g = row / DN;
    const T* wr = wuk + (int64_t)row * R;
    float acc[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) acc[t] = 0.f;
    for (int r = lane; r < R; r += 32) {
      const float w = ldf(wr, r);
#pragma unroll
      for (int t = 0; t < TT; ++t) acc[t] = fmaf(w, cs[t * R + r], acc[t]);
    }
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const float v = warp_sum(acc[t]);
      if (lane == 0) atomicAdd(&ssq[t * KV + g], v * v);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nt * KV; i += blockDim.x) {
    const int t = i / KV, g = i % KV;
    a.kscale[(int64_t)b * a.s_sb + (tb + t) * a.s_st + g] = rsqrtf(ssq[i] / (float)D + a.s.eps);
  }
}

// --- absorbed query --------------------------------------------------------
// grid: (KV, B, ceil(R / 64)); block 256.  One CTA per (group, batch row, 64
// latent columns).  The CTA's W_uk slice [DN x 64] is requested with every
// 16-byte load in flight at once, before waiting on the previous kernel
// (weights never come from it), and staged in shared memory in its own dtype.
// Thread (column pair, row slice of eight) accumulates its rows for four
// heads in registers; one shared-memory reduction over the slices finishes.
// The previous kernel is waited on before dependents are released, so the
// split kernel may fetch the cache as soon as it starts.
//   qt[b,h,r] = sum_i W_uk[g,i,r] * k_norm_w[i] * q[b,h,i]     (i < DN)
//   qr[b,h,:] = rope_{L-1}(q[b,h,DN:])                         (z-block 0 only)
constexpr int kAbsCols = 64, kAbsSlices = kThreads / 32, kAbsHB = 4;

template <typename T>
size_t absorb_smem_t(const b200mm_mla_shape& s) {
  const int hpg = s.H / s.KV, DN = s.D - s.DR;
  return sizeof(float) * ((size_t)hpg * s.D + (size_t)kAbsSlices * kAbsHB * kAbsCols) +
         sizeof(T) * (size_t)DN * kAbsCols + 16;
}
size_t absorb_smem_bytes(const b200mm_mla_shape& s) {
  return s.dtype == B200MM_F32 ? absorb_smem_t<float>(s) : absorb_smem_t<__half>(s);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) mla_absorb_kernel(const MlaDecodeArgs a, MlaWorkspace w) {
  MLA_SPAN(0, 0);
  extern __shared__ float sm[];
  const int H = a.s.H, KV = a.s.KV, D = a.s.D, DR = a.s.DR, DN = D - DR, R = a.s.R;
  const int hpg = H / KV, g = blockIdx.x, b = blockIdx.y, h0 = g * hpg, c0 = blockIdx.z * kAbsCols;
  float* qn = sm;                              // [hpg][D]  q, times k_norm_w on the first DN dims
  float* red = qn + hpg * D;                   // [slice][head][64]
  T* wsl = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(red + kAbsSlices * kAbsHB * kAbsCols) + 15) &
                                ~uintptr_t(15));  // [DN][64]
  float* ws = static_cast<float*>(a.ws);
  const T* wuk = static_cast<const T*>(a.w_uk) + (int64_t)g * DN * R;

  constexpr int VE = 16 / sizeof(T);  // elements per 16-byte load
  constexpr int U = 4;                // loads per thread per pass
  const bool vec = (R % VE) == 0 && c0 + kAbsCols <= R && ((reinterpret_cast<uintptr_t>(wuk) & 15u) == 0);
  const int per_row = kAbsCols / VE, total = DN * per_row;
  uint4 r[U];
  if (vec) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = u * kThreads + threadIdx.x;
      if (e < total) r[u] = *reinterpret_cast<const uint4*>(wuk + (int64_t)(e / per_row) * R + c0 + (e % per_row) * VE);
    }
  }
  pdl_wait();
  pdl_trigger();
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0)
    *reinterpret_cast<int*>(static_cast<unsigned char*>(a.ws) + w.off_err) = 0;
  if (vec) {
    for (int pass = 0; pass * U * kThreads < total; ++pass) {
      if (pass > 0) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int e = (pass * U + u) * kThreads + threadIdx.x;
          if (e < total)
            r[u] = *reinterpret_cast<const uint4*>(wuk + (int64_t)(e / per_row) * R + c0 + (e % per_row) * VE);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {  // row-major [DN][64]: consecutive threads, consecutive 16 bytes
        const int e = (pass * U + u) * kThreads + threadIdx.x;
        if (e < total) reinterpret_cast<uint4*>(wsl)[e] = r[u];
      }
    }
  } else {
    for (int e = threadIdx.x; e < DN * kAbsCols; e += blockDim.x) {
      const int i = e / kAbsCols, c = c0 + e % kAbsCols;
      wsl[e] = c < R ? wuk[(int64_t)i * R + c] : from_f<T>(0.f);
    }
  }
  const T* q = static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)h0 * D;
  for (int i = threadIdx.x; i < hpg * D; i += blockDim.x) {
    const int d = i % D;
    const float v = ldf(q, i);
    qn[i] = d < DN ? a.k_norm_w[d] * v : v;
  }
  __syncthreads();
  const int cp = threadIdx.x & 31, sl = threadIdx.x >> 5;  // columns 2cp, 2cp+1; rows sl, sl+8, ...
  float* qt = ws + w.off_qt / 4 + ((int64_t)b * H + h0) * R;
  for (int hb = 0; hb < hpg; hb += kAbsHB) {
    float acc[kAbsHB][2] = {};
    for (int i = sl; i < DN; i += kAbsSlices) {
      const float w0 = to_f<T>(wsl[i * kAbsCols + 2 * cp]), w1 = to_f<T>(wsl[i * kAbsCols + 2 * cp + 1]);
#pragma unroll
      for (int j = 0; j < kAbsHB; ++j) {
        if (hb + j >= hpg) break;
        const float qv = qn[(hb + j) * D + i];
        acc[j][0] = fmaf(w0, qv, acc[j][0]);
        acc[j][1] = fmaf(w1, qv, acc[j][1]);
      }
    }
#pragma unroll
    for (int j = 0; j < kAbsHB; ++j)
      *reinterpret_cast<float2*>(red + (sl * kAbsHB + j) * kAbsCols + 2 * cp) = make_float2(acc[j][0], acc[j][1]);
    __syncthreads();
    {
      const int j = threadIdx.x / kAbsCols, col = threadIdx.x % kAbsCols;
      if (hb + j < hpg && c0 + col < R) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < kAbsSlices; ++k) s += red[(k * kAbsHB + j) * kAbsCols + col];
        qt[(int64_t)(hb + j) * R + c0 + col] = s;
      }
    }
    __syncthreads();
  }
  MLA_SPAN(0, 1);
  if (blockIdx.z != 0) return;
  // qr = rope at position L-1 (rotate-half convention, angle = pos * inv_freq)
  const int half = DR / 2;
  const float pos = (float)a.qpos;
  float* qr = ws + w.off_qr / 4 + ((int64_t)b * H + h0) * DR;
  for (int o = threadIdx.x; o < hpg * DR; o += blockDim.x) {
    const int hq = o / DR, j = o % DR;
    const int i = j < half ? j : j - half;
    float sn, cs;
    sincosf(pos * a.inv_freq[i], &sn, &cs);
    const float* qh = qn + hq * D + DN;
    const float rot = j < half ? -qh[j + half] : qh[j - half];
    qr[o] = qh[j] * cs + rot * sn;
  }
}

// --- generic split kernel ---------------------------------------------------
// grid: (G); block 256.  CTA i walks its range of 64-token units, 16 tokens at
// a time, and writes one partial per batch row it touches.
// Shared: qt[H][R], qr[H][DR], acc[H][R], c[TT][R], z[TT][KV][DR], sc[H][TT],
// st[TT][KV], m[H], l[H], alpha[H].
template <typename T>
__global__ void __launch_bounds__(kThreads) mla_split_kernel(const MlaDecodeArgs a, MlaWorkspace w) {
  extern __shared__ float sm[];
  const int H = a.s.H, KV = a.s.KV, D = a.s.D, DR = a.s.DR, DN = D - DR, R = a.s.R;
  const int hpg = H / KV;
  const int cta = blockIdx.x;
  float* qt = sm;
  float* qr = qt + H * R;
  float* acc = qr + H * DR;
  float* cs = acc + H * R;
  float* z = cs + kTileT * R;
  float* sc = z + kTileT * KV * DR;
  float* st = sc + H * kTileT;
  float* mrun = st + kTileT * KV;
  float* lrun = mrun + H;
  float* alpha = lrun + H;

  float* ws = static_cast<float*>(a.ws);
  const int64_t u_begin = mla_range_begin(w, cta), u_end = mla_range_begin(w, cta + 1);

  pdl_trigger();
  pdl_wait();
  int64_t u = u_begin;
  while (u < u_end) {
    const int b = (int)(u / w.ntiles);
    const int64_t u_stop = imin64(u_end, (int64_t)(b + 1) * w.ntiles);  // units of row b in this range
    const T* c = static_cast<const T*>(a.c_kv) + (int64_t)b * a.c_sb;
    const T* kz = static_cast<const T*>(a.kz) + (int64_t)b * a.z_sb;
    const float* ks = a.kscale + (int64_t)b * a.s_sb;
    for (int i = threadIdx.x; i < H * R; i += blockDim.x) {
      qt[i] = ws[w.off_qt / 4 + (int64_t)b * H * R + i];
      acc[i] = 0.f;
    }
    for (int i = threadIdx.x; i < H * DR; i += blockDim.x) qr[i] = ws[w.off_qr / 4 + (int64_t)b * H * DR + i];
    for (int i = threadIdx.x; i < H; i += blockDim.x) { mrun[i] = -INFINITY; lrun[i] = 0.f; }
    __syncthreads();
    const int64_t t_begin = (u - (int64_t)b * w.ntiles) * kMlaUnit;
    const int64_t t_end = imin64(a.L, (u_stop - (int64_t)b * w.ntiles) * kMlaUnit);
    for (int64_t t0 = t_begin; t0 < t_end; t0 += kTileT) {
      const int nt = (int)imin64(kTileT, t_end - t0);
      for (int i = threadIdx.x; i < kTileT * R; i += blockDim.x) {
        const int t = i / R, r = i % R;
        cs[i] = t < nt ? ldf(c, (t0 + t) * a.c_st + r) : 0.f;
      }
      for (int i = threadIdx.x; i < kTileT * KV * DR; i += blockDim.x) {
        const int t = i / (KV * DR), rem = i % (KV * DR);
        z[i] = t < nt ? ldf(kz, (t0 + t) * a.z_st + rem) : 0.f;
      }
      for (int i = threadIdx.x; i < kTileT * KV; i += blockDim.x) {
        const int t = i / KV, g = i % KV;
        st[i] = t < nt ? ks[(t0 + t) * a.s_st + g] : 0.f;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < H * kTileT; i += blockDim.x) {
        const int h = i / kTileT, t = i % kTileT, g = h / hpg;
        float v = -INFINITY;
        if (t < nt) {
          float d0 = 0.f;
          for (int r = 0; r < R; ++r) d0 = fmaf(qt[h * R + r], cs[t * R + r], d0);
          for (int j = 0; j < DR; ++j) d0 = fmaf(qr[h * DR + j], z[(t * KV + g) * DR + j], d0);
          v = d0 * st[t * KV + g] * a.scale;
        }
        sc[i] = v;
      }
      __syncthreads();
      for (int h = threadIdx.x; h < H; h += blockDim.x) {
        float mx = mrun[h];
        for (int t = 0; t < nt; ++t) mx = fmaxf(mx, sc[h * kTileT + t]);
        const float al = expf(mrun[h] - mx);
        float sum = 0.f;
        for (int t = 0; t < kTileT; ++t) {
          const float p = t < nt ? expf(sc[h * kTileT + t] - mx) : 0.f;
          sc[h * kTileT + t] = p;
          sum += p;
        }
        lrun[h] = lrun[h] * al + sum;
        mrun[h] = mx;
        alpha[h] = al;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < H * R; i += blockDim.x) {
        const int h = i / R, r = i % R;
        float v = acc[i] * alpha[h];
        for (int t = 0; t < nt; ++t) v = fmaf(sc[h * kTileT + t], cs[t * R + r], v);
        acc[i] = v;
      }
      __syncthreads();
    }
    const int64_t slot = (int64_t)cta + b;
    float* pacc = ws + w.off_pacc / 4 + slot * H * R;
    float* pml = ws + w.off_pml / 4 + slot * H * 2;
    for (int i = threadIdx.x; i < H * R; i += blockDim.x) pacc[i] = acc[i];
    for (int h = threadIdx.x; h < H; h += blockDim.x) { pml[2 * h] = mrun[h]; pml[2 * h + 1] = lrun[h]; }
    __syncthreads();
    u = u_stop;
  }
}

// --- combine, step 1: merge the split partials ---------------------------
// grid: (H, B, rchunks); block 256.  Partials of row b: slot i + b for every
// range i overlapping [b*ntiles, (b+1)*ntiles).  Threads split the chunk's
// columns (float4 when R % 4 == 0) and the partials; the partial slices meet
// in shared memory.
//   av[b,h,:] = sum_k e^(m_k - M) acc_k / sum_k e^(m_k - M) l_k
template <typename V>
__device__ __forceinline__ void merge_cols(const float* pc, int64_t step, const float* wgt, int n, int width,
                                           float inv_l, float* av, float* red) {
  constexpr int VW = sizeof(V) / sizeof(float);
  const int nc = width / VW;
  if (nc <= 0) return;
  const int nps = nc >= (int)blockDim.x ? 1 : (int)blockDim.x / nc;
  const int ps = threadIdx.x / (nc >= (int)blockDim.x ? (int)blockDim.x : nc);
  if (nps == 1) {  // wide chunk: each thread owns columns, walks every partial
    for (int c = threadIdx.x; c < nc; c += blockDim.x) {
      float s[VW] = {};
      for (int k = 0; k < n; ++k) {
        const V p = *reinterpret_cast<const V*>(pc + k * step + c * VW);
        const float* pf = reinterpret_cast<const float*>(&p);
#pragma unroll
        for (int e = 0; e < VW; ++e) s[e] = fmaf(wgt[k], pf[e], s[e]);
      }
#pragma unroll
      for (int e = 0; e < VW; ++e) av[c * VW + e] = s[e] * inv_l;
    }
    return;
  }
  const int c = threadIdx.x % nc;
  if (ps < nps) {
    float s[VW] = {};
#pragma unroll 4
    for (int k = ps; k < n; k += nps) {
      const V p = *reinterpret_cast<const V*>(pc + k * step + c * VW);
      const float* pf = reinterpret_cast<const float*>(&p);
#pragma unroll
      for (int e = 0; e < VW; ++e) s[e] = fmaf(wgt[k], pf[e], s[e]);
    }
#pragma unroll
    for (int e = 0; e < VW; ++e) red[ps * width + c * VW + e] = s[e];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < width; o += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < nps; ++k) s += red[k * width + o];
    av[o] = s * inv_l;
  }
}

size_t merge_smem_bytes(const MlaWorkspace& w) { return sizeof(float) * (w.G + 2 + 4 * kThreads); }

template <typename T>
__global__ void __launch_bounds__(kThreads) mla_merge_kernel(const MlaDecodeArgs a, MlaWorkspace w) {
  MLA_SPAN(2, 0);
  extern __shared__ float sm[];
  const int H = a.s.H, R = a.s.R;
  const int h = blockIdx.x, b = blockIdx.y;
  const int r0 = blockIdx.z * w.rw, r1 = min(R, r0 + w.rw);
  const float* ws = static_cast<const float*>(a.ws);
  const float* pml = ws + w.off_pml / 4;
  const float* pacc = ws + w.off_pacc / 4;
  const int64_t lo = (int64_t)b * w.ntiles, hi = lo + w.ntiles;
  const int i0 = (int)(((lo + 1) * w.G - 1) / w.T);  // ranges overlapping [lo, hi)
  const int i1 = (int)((hi * w.G - 1) / w.T);
  const int n = i1 - i0 + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* wgt = sm;                 // [n]
  float* red = sm + w.G + 2;       // [partial slices][width], at most 4 * kThreads floats
  __shared__ float s_inv_l;

  pdl_trigger();
  pdl_wait();
  if (warp == 0) {
    float mx = -INFINITY;
    for (int k = lane; k < n; k += 32) mx = fmaxf(mx, pml[(((int64_t)i0 + k + b) * H + h) * 2]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float l = 0.f;
    for (int k = lane; k < n; k += 32) {
      const float* p = pml + (((int64_t)i0 + k + b) * H + h) * 2;
      const float e = expf(p[0] - mx);
      wgt[k] = e;
      l += e * p[1];
    }
    l = warp_sum(l);
    if (lane == 0) {
      s_inv_l = 1.f / l;
      if (a.ml_out && blockIdx.z == 0) {
        // a split kernel that gave up on a bounded wait poisons the partial
        // (NaN propagates through the cross-range merge), as the combine
        // step does for a whole decode
        const bool failed = *reinterpret_cast<const int*>(reinterpret_cast<const unsigned char*>(ws) + w.off_err) != 0;
        a.ml_out[((int64_t)b * H + h) * 2] = failed ? __int_as_float(0x7fc00000) : mx;
        a.ml_out[((int64_t)b * H + h) * 2 + 1] = l;
      }
    }
  }
  __syncthreads();
  const int64_t step = (int64_t)H * R;
  const float* pc = pacc + (((int64_t)i0 + b) * H + h) * R + r0;
  float* av = (a.av_out ? a.av_out : const_cast<float*>(ws) + w.off_av / 4) + ((int64_t)b * H + h) * R + r0;
  if ((R & 3) == 0)
    merge_cols<float4>(pc, step, wgt, n, r1 - r0, s_inv_l, av, red);
  else
    merge_cols<float>(pc, step, wgt, n, r1 - r0, s_inv_l, av, red);
  MLA_SPAN(2, 1);
}

// --- combine, step 2: out[b,h,d] = W_uv[g,d,:] . av[b,h,:] ------------------
// grid: (KV, B, ceil(D / 32)); block 256.  One CTA per (group, row, 32 output
// dims).  The 32 W_uv rows are staged in shared memory (row pitch padded by
// one word, so lane-per-row reads hit 32 different banks) with every load in flight
// before waiting on the previous kernel; lane = output dim, warp w sums
// latent slice [R*w/8, R*(w+1)/8) for up to four heads at once, and one
// shared-memory reduction over the warps finishes.
constexpr int kCombDims = 32, kCombHB = 4;

template <typename T>
size_t combine_smem_t(const b200mm_mla_shape& s) {
  const int hpg = s.H / s.KV;
  const size_t pitch = (size_t)s.R * sizeof(T) + 4;
  return sizeof(float) * ((size_t)hpg * s.R + (size_t)(kThreads / 32) * kCombHB * kCombDims) + kCombDims * pitch + 16;
}
size_t combine_smem_bytes(const b200mm_mla_shape& s) {
  return s.dtype == B200MM_F32 ? combine_smem_t<float>(s) : combine_smem_t<__half>(s);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) mla_combine_kernel(const MlaDecodeArgs a, MlaWorkspace w) {
  MLA_SPAN(3, 0);
  extern __shared__ float4 sm4[];
  const int H = a.s.H, KV = a.s.KV, D = a.s.D, R = a.s.R;
  const int hpg = H / KV, g = blockIdx.x, b = blockIdx.y, h0 = g * hpg, d0 = blockIdx.z * kCombDims;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NWp = kThreads / 32;
  float* av = reinterpret_cast<float*>(sm4);   // [hpg][R]
  float* red = av + hpg * R;                   // [warp][head][dim]
  unsigned char* wrows = reinterpret_cast<unsigned char*>(red + NWp * kCombHB * kCombDims);
  const int pitch = R * (int)sizeof(T) + 4;    // bytes per staged W_uv row (4-byte aligned)
  const T* wuv = static_cast<const T*>(a.w_uv) + (int64_t)g * D * R;
  constexpr int VE = 16 / sizeof(T);
  const bool vec = (R % VE) == 0 && ((reinterpret_cast<uintptr_t>(wuv) & 15u) == 0);
  const int per_row = R / VE, nrows = min(kCombDims, D - d0), total = nrows * per_row;
  constexpr int U = 4;
  uint4 r[U];
  if (vec) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = u * kThreads + threadIdx.x;
      if (e < total) r[u] = *reinterpret_cast<const uint4*>(wuv + (int64_t)(d0 + e / per_row) * R + (e % per_row) * VE);
    }
  }
  pdl_trigger();
  pdl_wait();
  if (vec) {
    for (int pass = 0; pass * U * kThreads < total; ++pass) {
      if (pass > 0) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int e = (pass * U + u) * kThreads + threadIdx.x;
          if (e < total)
            r[u] = *reinterpret_cast<const uint4*>(wuv + (int64_t)(d0 + e / per_row) * R + (e % per_row) * VE);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int e = (pass * U + u) * kThreads + threadIdx.x;
        if (e < total) {
          uint32_t* dst = reinterpret_cast<uint32_t*>(wrows + (e / per_row) * pitch + (e % per_row) * 16);
          dst[0] = r[u].x;
          dst[1] = r[u].y;
          dst[2] = r[u].z;
          dst[3] = r[u].w;
        }
      }
    }
  } else {
    for (int e = threadIdx.x; e < nrows * R; e += blockDim.x)
      reinterpret_cast<T*>(wrows + (e / R) * pitch)[e % R] = wuv[(int64_t)(d0 + e / R) * R + e % R];
  }
  const float* src = static_cast<const float*>(a.ws) + w.off_av / 4 + ((int64_t)b * H + h0) * R;
  for (int o = threadIdx.x; o < hpg * R; o += blockDim.x) av[o] = src[o];
  __syncthreads();
  // a split kernel that gave up on a bounded wait leaves NaN, never a silent result
  const bool failed = *reinterpret_cast<const int*>(static_cast<const unsigned char*>(a.ws) + w.off_err) != 0;
  const int r0 = (int)((int64_t)R * warp / NWp), r1 = (int)((int64_t)R * (warp + 1) / NWp);
  const T* wr = reinterpret_cast<const T*>(wrows + lane * pitch);
  for (int hb = 0; hb < hpg; hb += kCombHB) {
    float v[kCombHB] = {};
    if (lane < nrows) {
      int rr = r0;
      if (sizeof(T) == 2) {  // pairs: one 4-byte read per lane (r0 is even when R % 16 == 0)
        for (; (r0 & 1) == 0 && rr + 1 < r1; rr += 2) {
          const uint32_t pr = *reinterpret_cast<const uint32_t*>(wr + rr);
          const T* pe = reinterpret_cast<const T*>(&pr);
          const float w0 = to_f<T>(pe[0]), w1 = to_f<T>(pe[1]);
#pragma unroll
          for (int j = 0; j < kCombHB; ++j) {
            if (hb + j >= hpg) break;
            const float2 x = *reinterpret_cast<const float2*>(av + (hb + j) * R + rr);
            v[j] = fmaf(w0, x.x, fmaf(w1, x.y, v[j]));
          }
        }
      }
      for (; rr < r1; ++rr) {
        const float wv = to_f<T>(wr[rr]);
#pragma unroll
        for (int j = 0; j < kCombHB; ++j)
          if (hb + j < hpg) v[j] = fmaf(wv, av[(hb + j) * R + rr], v[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < kCombHB; ++j) red[(warp * kCombHB + j) * kCombDims + lane] = v[j];
    __syncthreads();
    if (threadIdx.x < kCombHB * kCombDims) {
      const int j = threadIdx.x / kCombDims, dd = threadIdx.x % kCombDims;
      if (hb + j < hpg && dd < nrows) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < NWp; ++k) s += red[(k * kCombHB + j) * kCombDims + dd];
        T* out = static_cast<T*>(a.out) + (int64_t)b * a.o_sb + (int64_t)(h0 + hb + j) * D;
        out[d0 + dd] = from_f<T>(failed ? __int_as_float(0x7fc00000) : s);
      }
    }
    __syncthreads();
  }
  MLA_SPAN(3, 1);
}

size_t split_smem_bytes(const b200mm_mla_shape& s) {
  const int H = s.H, R = s.R, DR = s.DR, KV = s.KV;
  return sizeof(float) * ((size_t)H * R * 2 + (size_t)H * DR + (size_t)kTileT * R +
                          (size_t)kTileT * KV * DR + (size_t)H * kTileT + (size_t)kTileT * KV + 3 * H);
}

template <typename K, typename... Args>
int launch_smem(K kern, dim3 grid, size_t smem, cudaStream_t st, Args... args) {
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return B200MM_ERR_LAUNCH;
  }
  return launch_pdl(kern, grid, dim3(kThreads), smem, st, args...) == cudaSuccess ? B200MM_OK
                                                                                  : B200MM_ERR_LAUNCH;
}

template <typename T>
int decode_t(const MlaDecodeArgs& a) {
  MlaMaps maps;
  const bool fast =
      !g_force_generic.load(std::memory_order_relaxed) && mla_fast_supported(a) && mla_fast_maps(a, &maps);
  const MlaWorkspace w = mla_plan(a.s, a.L, fast);
  const int B = a.s.B, H = a.s.H;
  int st = launch_smem(mla_absorb_kernel<T>, dim3(a.s.KV, B, (a.s.R + kAbsCols - 1) / kAbsCols),
                       absorb_smem_bytes(a.s), a.stream, a, w);
  if (st) return st;
  if (fast) {
    st = mla_tc_split_launch(a, w, maps);
  } else {
    st = launch_smem(mla_split_kernel<T>, dim3(w.G), split_smem_bytes(a.s), a.stream, a, w);
  }
  if (st) return st;
  st = launch_smem(mla_merge_kernel<T>, dim3(H, B, w.rchunks), merge_smem_bytes(w), a.stream, a, w);
  if (st) return st;
  if (a.av_out) return B200MM_OK;  // a partial decode stops at the range's merged latent
  return launch_smem(mla_combine_kernel<T>, dim3(a.s.KV, B, (a.s.D + kCombDims - 1) / kCombDims),
                     combine_smem_bytes(a.s), a.stream, a, w);
}

// --- merge of per-range partials (a context split across GPUs) --------------
// grid: (H, B); block 256.  Range r covered its tokens with max score m_r and
// sum of exp s_r and left av_r normalised over them:
//   av[b,h,:] = sum_r s_r e^(m_r - M) av_r / sum_r s_r e^(m_r - M),  M = max_r m_r
__global__ void __launch_bounds__(kThreads) mla_rank_merge_kernel(const MlaDecodeArgs a, MlaWorkspace w,
                                                                  const float* __restrict__ avp, int64_t avs,
                                                                  const float* __restrict__ mlp, int64_t mls,
                                                                  int n) {
  const int H = a.s.H, R = a.s.R;
  const int h = blockIdx.x, b = blockIdx.y;
  __shared__ float wgt[64];
  pdl_trigger();
  pdl_wait();
  // the W_uv step that follows checks this workspace's error flag: nothing
  // here waits, so it is clear (a failed range already carries NaN)
  if (h == 0 && b == 0 && threadIdx.x == 0)
    *reinterpret_cast<int*>(static_cast<unsigned char*>(a.ws) + w.off_err) = 0;
  if (threadIdx.x < 32) {
    float mx = -INFINITY;
    for (int r = threadIdx.x; r < n; r += 32) mx = fmaxf(mx, mlp[r * mls + ((int64_t)b * H + h) * 2]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float tot = 0.f;
    for (int r = threadIdx.x; r < n; r += 32) {
      const float* p = mlp + r * mls + ((int64_t)b * H + h) * 2;
      const float e = p[1] > 0.f ? p[1] * expf(p[0] - mx) : 0.f;
      wgt[r] = e;
      tot += e;
    }
    tot = warp_sum(tot);
    for (int r = threadIdx.x; r < n; r += 32) wgt[r] /= tot;
  }
  __syncthreads();
  float* av = static_cast<float*>(a.ws) + w.off_av / 4 + ((int64_t)b * H + h) * R;
  for (int c = threadIdx.x; c < R; c += blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < n; ++r) s = fmaf(wgt[r], avp[r * avs + ((int64_t)b * H + h) * R + c], s);
    av[c] = s;
  }
}

template <typename T>
int combine_partials_t(const MlaDecodeArgs& a, const float* avp, int64_t avs, const float* mlp, int64_t mls, int n) {
  const MlaWorkspace w = mla_plan(a.s, 1, false);
  int st = launch_pdl(mla_rank_merge_kernel, dim3(a.s.H, a.s.B), dim3(kThreads), 0, a.stream, a, w, avp, avs, mlp,
                      mls, n) == cudaSuccess
               ? B200MM_OK
               : B200MM_ERR_LAUNCH;
  if (st) return st;
  return launch_smem(mla_combine_kernel<T>, dim3(a.s.KV, a.s.B, (a.s.D + kCombDims - 1) / kCombDims),
                     combine_smem_bytes(a.s), a.stream, a, w);
}

template <typename T>
int append_t(const MlaAppendArgs& a) {
  const int64_t n = a.t1 - a.t0;
  dim3 grid((unsigned)((n + 7) / 8), (unsigned)a.s.B);
  const size_t smem = sizeof(float) * (8 * (size_t)a.s.R + 8 * (size_t)a.s.KV);
  return launch_smem(mla_append_kernel<T>, grid, smem, a.stream, a);
}

}  // namespace

int mla_validate_shape(const b200mm_mla_shape& s) {
  if (s.dtype != B200MM_F32 && s.dtype != B200MM_F16 && s.dtype != B200MM_BF16) return B200MM_ERR_DTYPE;
  if (s.B < 0 || s.B > 65535 || s.H < 1 || s.KV < 1 || s.H % s.KV || s.H > 65535) return B200MM_ERR_SHAPE;
  if (s.D < 1 || s.D > 1024 || s.DR < 0 || s.DR > s.D || (s.DR & 1)) return B200MM_ERR_SHAPE;
  if (s.R < 1 || s.R > 4096) return B200MM_ERR_SHAPE;
  if (!(s.eps >= 0.f)) return B200MM_ERR_ARG;
  if (split_smem_bytes(s) > 200 * 1024 || absorb_smem_bytes(s) > 200 * 1024) return B200MM_ERR_SHAPE;
  if (combine_smem_bytes(s) > 200 * 1024) return B200MM_ERR_SHAPE;
  return B200MM_OK;
}

MlaWorkspace mla_plan(const b200mm_mla_shape& s, int64_t L, bool fast) {
  MlaWorkspace w{};
  const int B = s.B > 0 ? s.B : 1;
  w.ntiles = (L + kMlaUnit - 1) / kMlaUnit;
  w.T = (int64_t)B * w.ntiles;
  const int64_t want = fast ? mla_fast_ctas() : num_sms(current_device());
  w.G = (int)(want < w.T ? want : w.T);
  const size_t BH = (size_t)B * s.H;
  const size_t slots = (size_t)w.G + B;
  w.off_qt = 0;
  w.off_qr = align256(w.off_qt + sizeof(float) * BH * s.R);
  w.off_pacc = align256(w.off_qr + sizeof(float) * BH * (s.DR > 0 ? s.DR : 1));
  w.off_pml = align256(w.off_pacc + sizeof(float) * slots * s.H * s.R);
  w.off_av = align256(w.off_pml + sizeof(float) * slots * s.H * 2);
  w.off_err = align256(w.off_av + sizeof(float) * BH * s.R);
  // merge parallelism: about 16 partials per CTA, latent chunks of >= 32
  const int64_t parts = (w.G + B - 1) / B + 1;
  const int rc = (int)((parts + 15) / 16), max_rc = (s.R + 31) / 32;
  w.rchunks = rc < 1 ? 1 : (rc > max_rc ? max_rc : rc);
  w.rw = (s.R + w.rchunks - 1) / w.rchunks;
  if ((s.R & 3) == 0) w.rw = (w.rw + 3) & ~3;  // float4 columns in the merge
  w.rchunks = (s.R + w.rw - 1) / w.rw;
  w.total = align256(w.off_err + 16);
  return w;
}

size_t mla_workspace_bytes(const b200mm_mla_shape& s, int64_t L) {
  const size_t a = mla_plan(s, L, true).total, b = mla_plan(s, L, false).total;
  return a > b ? a : b;
}

int mla_append_launch(const MlaAppendArgs& a) {
  if (!g_force_generic.load(std::memory_order_relaxed) && mla_fill_tc_supported(a)) return mla_fill_tc_launch(a);
  if (a.s.dtype == B200MM_BF16) return append_t<__nv_bfloat16>(a);
  if (a.s.dtype == B200MM_F16) return append_t<__half>(a);
  return append_t<float>(a);
}

int mla_combine_partials_launch(const MlaDecodeArgs& a, const float* av_parts, int64_t av_stride,
                                const float* ml_parts, int64_t ml_stride, int nparts) {
  if (a.s.dtype == B200MM_BF16) return combine_partials_t<__nv_bfloat16>(a, av_parts, av_stride, ml_parts, ml_stride, nparts);
  if (a.s.dtype == B200MM_F16) return combine_partials_t<__half>(a, av_parts, av_stride, ml_parts, ml_stride, nparts);
  return combine_partials_t<float>(a, av_parts, av_stride, ml_parts, ml_stride, nparts);
}

int mla_decode_launch(const MlaDecodeArgs& a) {
  if (a.s.dtype == B200MM_BF16) return decode_t<__nv_bfloat16>(a);
  if (a.s.dtype == B200MM_F16) return decode_t<__half>(a);
  return decode_t<float>(a);
}

}  // namespace b200mm
