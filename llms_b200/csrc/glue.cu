// The decode step's small ops around the projections, one launch each instead
// of the engine's chains of elementwise torch kernels:
//
//   b200mm_rmsnorm      y = w * cast(x * rsqrt(mean(x^2) + eps)), optionally
//                       on h = cast(x + r) (the residual add before a norm),
//                       h stored too  -- engine/attention.py:20-33 and the
//                       residual adds of engine/model.py:54-63;
//   b200mm_qk_norm_rope q = rope(q_norm(q)), k = rope(k_norm(k)) for one new
//                       token per row, straight from the fused projection's
//                       output, with k and v written into the KV cache at the
//                       token's position -- engine/attention.py:119-131.
//
// Both keep the engine's rounding points exactly: the norm computes in fp32
// and casts to the activation dtype before the weight multiply; RoPE is
// x * cos + rotate_half(x) * sin with cos / sin cast to the activation dtype
// and each product and the sum rounded to it.  Only the fp32 summation order
// of the mean differs from torch.
#include "dense.cuh"

namespace b200mm {

namespace {

template <typename T>
__device__ __forceinline__ float rnd(float v) {
  return to_f<T>(from_f<T>(v));
}

// One CTA per row; 16-byte vectors; N % (8 for 16-bit, 4 for fp32) == 0.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ r,
                                                       int64_t ldr, T* __restrict__ h, int64_t ldh,
                                                       const T* __restrict__ w, T* __restrict__ y, int64_t ldy, int N,
                                                       float eps) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float red[8];
  const int64_t m = blockIdx.x;
  const T* xr = x + m * ldx;
  const T* rr = r ? r + m * ldr : nullptr;
  pdl_trigger();
  pdl_wait();
  // at most 8 vectors per thread held in registers (N <= 256 * 8 * V)
  constexpr int MAXV = 8;
  float v[MAXV][V];
  float ss = 0.f;
  const int nv = N / V;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nv) {
      Chunk<T>::unpack(*reinterpret_cast<const uint4*>(xr + (int64_t)c * V), v[i]);
      if (rr) {
        float t[V];
        Chunk<T>::unpack(*reinterpret_cast<const uint4*>(rr + (int64_t)c * V), t);
#pragma unroll
        for (int e = 0; e < V; ++e) v[i][e] = rnd<T>(v[i][e] + t[e]);
        if (h) {
          T o[V];
#pragma unroll
          for (int e = 0; e < V; ++e) o[e] = from_f<T>(v[i][e]);
          *reinterpret_cast<uint4*>(h + m * ldh + (int64_t)c * V) = *reinterpret_cast<const uint4*>(o);
        }
      }
#pragma unroll
      for (int e = 0; e < V; ++e) ss = fmaf(v[i][e], v[i][e], ss);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)N + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nv) {
      float wf[V];
      Chunk<T>::unpack(*reinterpret_cast<const uint4*>(w + (int64_t)c * V), wf);
      T o[V];
#pragma unroll
      for (int e = 0; e < V; ++e) o[e] = from_f<T>(wf[e] * rnd<T>(v[i][e] * inv));
      *reinterpret_cast<uint4*>(y + m * ldy + (int64_t)c * V) = *reinterpret_cast<const uint4*>(o);
    }
  }
}

// One warp per (row, head) of q, k and v: E = D / 32 elements per lane
// (lane l holds [E*l, E*l + E)); rotate_half pairs element j with j +- D/2,
// which sits 16 lanes away.
template <typename T, int E>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const T* __restrict__ qkv, int64_t ldq, int H, int KV, const T* __restrict__ qw, const T* __restrict__ kw,
    const T* __restrict__ cos_t, const T* __restrict__ sin_t, int64_t pos_host,
    const int64_t* __restrict__ pos_dev, T* __restrict__ q_out, int64_t q_sb, int64_t q_sh, T* __restrict__ kc,
    int64_t k_sb, int64_t k_sh, int64_t k_st, T* __restrict__ vc, int64_t v_sb, int64_t v_sh, int64_t v_st, int B,
    float eps) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int per_row = H + 2 * KV;
  pdl_trigger();
  pdl_wait();
  if (gw >= B * per_row) return;
  const int b = gw / per_row, hd = gw % per_row;
  const int64_t pos = pos_dev ? *pos_dev : pos_host;
  const T* src = qkv + (int64_t)b * ldq + (int64_t)hd * D + E * lane;
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = to_f<T>(src[e]);
  if (hd >= H + KV) {  // v: straight into the cache
    T* dst = vc + (int64_t)b * v_sb + (int64_t)(hd - H - KV) * v_sh + pos * v_st + E * lane;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = from_f<T>(x[e]);
    return;
  }
  const bool isq = hd < H;
  const T* w = isq ? qw : kw;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) ss = fmaf(x[e], x[e], ss);
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
  float n[E];
#pragma unroll
  for (int e = 0; e < E; ++e) n[e] = rnd<T>(to_f<T>(w[E * lane + e]) * rnd<T>(x[e] * inv));
  const bool lo = lane < 16;
  float out[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float other = __shfl_xor_sync(0xffffffffu, n[e], 16);
    const float rot = lo ? -other : other;  // rotate_half: [-x2, x1]
    const int j = E * lane + e;
    const float c = to_f<T>(cos_t[pos * D + j]), s = to_f<T>(sin_t[pos * D + j]);
    out[e] = rnd<T>(rnd<T>(n[e] * c) + rnd<T>(rot * s));
  }
  T* dst = isq ? q_out + (int64_t)b * q_sb + (int64_t)hd * q_sh + E * lane
               : kc + (int64_t)b * k_sb + (int64_t)(hd - H) * k_sh + pos * k_st + E * lane;
#pragma unroll
  for (int e = 0; e < E; ++e) dst[e] = from_f<T>(out[e]);
}

template <typename T>
int rmsnorm_t(const void* x, int64_t ldx, const void* r, int64_t ldr, void* h, int64_t ldh, const void* w, void* y,
              int64_t ldy, int M, int N, float eps, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  if (N % V || N > 256 * 8 * V) return B200MM_ERR_SHAPE;
  auto al = [](const void* p) { return ((uintptr_t)p & 15u) == 0; };
  if (!al(x) || !al(w) || !al(y) || (r && !al(r)) || (h && !al(h))) return B200MM_ERR_ALIGN;
  if ((ldx * sizeof(T)) % 16 || (ldy * sizeof(T)) % 16 || (r && (ldr * sizeof(T)) % 16) ||
      (h && (ldh * sizeof(T)) % 16))
    return B200MM_ERR_ALIGN;
  int threads = (N / V + 31) / 32 * 32;
  if (threads > 256) threads = 256;
  return launch_pdl(rmsnorm_kernel<T>, dim3(M), dim3(threads), 0, st, static_cast<const T*>(x), ldx,
                    static_cast<const T*>(r), ldr, static_cast<T*>(h), ldh, static_cast<const T*>(w),
                    static_cast<T*>(y), ldy, N, eps) == cudaSuccess
             ? B200MM_OK
             : B200MM_ERR_LAUNCH;
}

template <typename T, int E>
int qkr_t(const void* qkv, int64_t ldq, int B, int H, int KV, const void* qw, const void* kw, const void* cos_t,
          const void* sin_t, int64_t pos, const int64_t* pos_dev, void* q_out, int64_t q_sb, int64_t q_sh, void* kc,
          int64_t k_sb, int64_t k_sh, int64_t k_st, void* vc, int64_t v_sb, int64_t v_sh, int64_t v_st, float eps,
          cudaStream_t st) {
  const int warps = B * (H + 2 * KV);
  const int blocks = (warps + 7) / 8;
  return launch_pdl(qk_norm_rope_kernel<T, E>, dim3(blocks), dim3(256), 0, st, static_cast<const T*>(qkv), ldq, H,
                    KV, static_cast<const T*>(qw), static_cast<const T*>(kw), static_cast<const T*>(cos_t),
                    static_cast<const T*>(sin_t), pos, pos_dev,
                    static_cast<T*>(q_out), q_sb, q_sh, static_cast<T*>(kc), k_sb, k_sh, k_st, static_cast<T*>(vc),
                    v_sb, v_sh, v_st, B, eps) == cudaSuccess
             ? B200MM_OK
             : B200MM_ERR_LAUNCH;
}

template <typename T>
int qkr_d(int D, const void* qkv, int64_t ldq, int B, int H, int KV, const void* qw, const void* kw,
          const void* cos_t, const void* sin_t, int64_t pos, const int64_t* pos_dev, void* q_out, int64_t q_sb,
          int64_t q_sh, void* kc, int64_t k_sb, int64_t k_sh, int64_t k_st, void* vc, int64_t v_sb, int64_t v_sh,
          int64_t v_st, float eps, cudaStream_t st) {
  if (D == 64)
    return qkr_t<T, 2>(qkv, ldq, B, H, KV, qw, kw, cos_t, sin_t, pos, pos_dev, q_out, q_sb, q_sh, kc, k_sb, k_sh,
                       k_st, vc, v_sb, v_sh, v_st, eps, st);
  if (D == 128)
    return qkr_t<T, 4>(qkv, ldq, B, H, KV, qw, kw, cos_t, sin_t, pos, pos_dev, q_out, q_sb, q_sh, kc, k_sb, k_sh,
                       k_st, vc, v_sb, v_sh, v_st, eps, st);
  if (D == 256)
    return qkr_t<T, 8>(qkv, ldq, B, H, KV, qw, kw, cos_t, sin_t, pos, pos_dev, q_out, q_sb, q_sh, kc, k_sb, k_sh,
                       k_st, vc, v_sb, v_sh, v_st, eps, st);
  return B200MM_ERR_SHAPE;
}

}  // namespace

int glue_rmsnorm(const void* x, int64_t ldx, const void* r, int64_t ldr, void* h, int64_t ldh, const void* w, void* y,
                 int64_t ldy, int M, int N, float eps, int dtype, cudaStream_t st) {
  if (dtype == B200MM_BF16) return rmsnorm_t<__nv_bfloat16>(x, ldx, r, ldr, h, ldh, w, y, ldy, M, N, eps, st);
  if (dtype == B200MM_F16) return rmsnorm_t<__half>(x, ldx, r, ldr, h, ldh, w, y, ldy, M, N, eps, st);
  if (dtype == B200MM_F32) return rmsnorm_t<float>(x, ldx, r, ldr, h, ldh, w, y, ldy, M, N, eps, st);
  return B200MM_ERR_DTYPE;
}

int glue_qk_norm_rope(const void* qkv, int64_t ldq, int B, int H, int KV, int D, const void* qw, const void* kw,
                      const void* cos_t, const void* sin_t, int64_t pos, const int64_t* pos_dev, void* q_out,
                      int64_t q_sb, int64_t q_sh, void* kc, int64_t k_sb, int64_t k_sh, int64_t k_st, void* vc,
                      int64_t v_sb, int64_t v_sh, int64_t v_st, float eps, int dtype, cudaStream_t st) {
  if (dtype == B200MM_BF16)
    return qkr_d<__nv_bfloat16>(D, qkv, ldq, B, H, KV, qw, kw, cos_t, sin_t, pos, pos_dev, q_out, q_sb, q_sh, kc,
                                k_sb, k_sh, k_st, vc, v_sb, v_sh, v_st, eps, st);
  if (dtype == B200MM_F16)
    return qkr_d<__half>(D, qkv, ldq, B, H, KV, qw, kw, cos_t, sin_t, pos, pos_dev, q_out, q_sb, q_sh, kc, k_sb, k_sh,
                         k_st, vc, v_sb, v_sh, v_st, eps, st);
  if (dtype == B200MM_F32)
    return qkr_d<float>(D, qkv, ldq, B, H, KV, qw, kw, cos_t, sin_t, pos, pos_dev, q_out, q_sb, q_sh, kc, k_sb, k_sh,
                        k_st, vc, v_sb, v_sh, v_st, eps, st);
  return B200MM_ERR_DTYPE;
}

}  // namespace b200mm
