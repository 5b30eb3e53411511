// General projection kernel: 64x64 output tiles on CUDA cores, any shape,
// any row stride, any alignment.  It serves what the specialised kernels
// decline (odd K, unaligned rows, fp32 at M > 8, int8 at M > 8) and is the
// cross-check for them in the tests.  Scalar loads, fp32 accumulate.
#include "dense.cuh"

namespace b200mm {

namespace {

constexpr int BM = 64, BN = 64, BK = 16;

struct TiledParams {
  const void* x; int64_t ldx;
  const void* w0; int64_t ldw0;
  const void* w1; int64_t ldw1;
  const float* s0; const float* s1;
  void* y; int64_t ldy;
  int M, N, K;
};

template <typename TX, typename TW, bool GATE>
__global__ void __launch_bounds__(256) tiled_kernel(const TiledParams p) {
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[GATE ? 2 : 1][BK][BN + 4];

  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const TX* x = static_cast<const TX*>(p.x);
  const TW* w0 = static_cast<const TW*>(p.w0);
  const TW* w1 = static_cast<const TW*>(p.w1);

  pdl_trigger();
  pdl_wait();

  float acc[GATE ? 2 : 1][4][4];
#pragma unroll
  for (int g = 0; g < (GATE ? 2 : 1); ++g)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[g][i][j] = 0.f;

  for (int k0 = 0; k0 < p.K; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      const int mm = i / BK, kk = i % BK;
      const int m = m0 + mm, k = k0 + kk;
      xs[kk][mm] = (m < p.M && k < p.K) ? to_f<TX>(x[(int64_t)m * p.ldx + k]) : 0.f;
    }
    for (int i = threadIdx.x; i < BN * BK; i += 256) {
      const int nn = i / BK, kk = i % BK;
      const int n = n0 + nn, k = k0 + kk;
      const bool ok = n < p.N && k < p.K;
      ws[0][kk][nn] = ok ? to_f<TW>(w0[(int64_t)n * p.ldw0 + k]) : 0.f;
      if (GATE) ws[GATE ? 1 : 0][kk][nn] = ok ? to_f<TW>(w1[(int64_t)n * p.ldw1 + k]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[GATE ? 2 : 1][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int g = 0; g < (GATE ? 2 : 1); ++g)
#pragma unroll
        for (int j = 0; j < 4; ++j) b[g][j] = ws[g][kk][tx * 4 + j];
#pragma unroll
      for (int g = 0; g < (GATE ? 2 : 1); ++g)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[g][i][j] = fmaf(a[i], b[g][j], acc[g][i][j]);
    }
    __syncthreads();
  }

  TX* y = static_cast<TX*>(p.y);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= p.N) continue;
      float v;
      if (GATE) {
        float g = acc[0][i][j], u = acc[GATE ? 1 : 0][i][j];
        if (p.s0) { g *= p.s0[n]; u *= p.s1[n]; }
        v = silu_mul(g, u);
      } else {
        v = acc[0][i][j];
        if (p.s0) v *= p.s0[n];
      }
      y[(int64_t)m * p.ldy + n] = from_f<TX>(v);
    }
  }
}

template <typename TX, typename TW>
int launch_t(const DenseArgs& a) {
  TiledParams p{a.x, a.ldx, a.w0, a.ldw0, a.w1, a.ldw1, a.s0, a.s1, a.y, a.ldy, a.M, a.N, a.K};
  dim3 grid((a.N + BN - 1) / BN, (a.M + BM - 1) / BM);
  if (grid.y > 65535) return B200MM_ERR_SHAPE;
  cudaError_t e = a.gate ? launch_pdl(tiled_kernel<TX, TW, true>, grid, dim3(256), 0, a.stream, p)
                         : launch_pdl(tiled_kernel<TX, TW, false>, grid, dim3(256), 0, a.stream, p);
  return e == cudaSuccess ? B200MM_OK : B200MM_ERR_LAUNCH;
}

}  // namespace

int tiled_launch(const DenseArgs& a) {
  if (a.w8) {
    if (a.dtype == B200MM_BF16) return launch_t<__nv_bfloat16, int8_t>(a);
    if (a.dtype == B200MM_F16) return launch_t<__half, int8_t>(a);
    return B200MM_ERR_DTYPE;
  }
  if (a.dtype == B200MM_BF16) return launch_t<__nv_bfloat16, __nv_bfloat16>(a);
  if (a.dtype == B200MM_F16) return launch_t<__half, __half>(a);
  if (a.dtype == B200MM_F32) return launch_t<float, float>(a);
  return B200MM_ERR_DTYPE;
}

}  // namespace b200mm
