// Shared device/host helpers for the b200mm kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <atomic>

#include "../../include/b200mm.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "b200mm is built for sm_100a only"
#endif

namespace b200mm {

// ---------------------------------------------------------------------------
// host-side bookkeeping
// ---------------------------------------------------------------------------
extern std::atomic<uint64_t> g_launches;
extern std::atomic<int> g_force_generic;  // tests: route every call to the generic kernels
inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int num_sms(int device);          // cached multiprocessor count of `device`
int current_device();             // cudaGetDevice with caching of nothing

// peer.cu: column-block all-gather over peer memory (b200mm_peer_gather)
int peer_gather_launch(const void* src, int64_t ld_src, int64_t rows, const int64_t* widths, int nparts,
                       void* const* dst, int64_t ld_dst, int elem_bytes, int rank, int world, unsigned* const* flags,
                       unsigned* seen, int* err, int nctas, cudaStream_t stream);

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? B200MM_OK : B200MM_ERR_LAUNCH;
}

// Launch `kernel` with programmatic dependent launch enabled, so its prologue
// (weight prefetch) may overlap the tail of the previous kernel on the stream.
// The kernel must execute `griddepcontrol.wait` before touching data another
// kernel produced or consumes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl for a kernel in thread-block clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t stream, int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
// thread-block clusters: rank, distributed shared memory, cluster-wide barrier
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(out)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(rank));
  return out;
}
__device__ __forceinline__ void st_cluster_f2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void st_cluster_f4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// int8 pair (bytes 2j, 2j+1 of the sign-flipped word w ^ 0x80808080) -> fp16x2,
// exact: the bytes become the low mantissa bits of 1024 + (q + 128), and
// subtracting 1152 leaves q.
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t wflip, int j) {
  const uint32_t h = __byte_perm(wflip, 0x64646464u, j == 0 ? 0x4140u : 0x4342u);
  const __half2 v =
      __hsub2(*reinterpret_cast<const __half2*>(&h), __half2(__float2half(1152.f), __float2half(1152.f)));
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// 16-byte streaming load: read-only, not kept in L1, 256-byte L2 sector prefetch.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

template <typename T> struct ElemTraits;
template <> struct ElemTraits<float> {
  static constexpr int kCode = B200MM_F32;
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};
template <> struct ElemTraits<__half> {
  static constexpr int kCode = B200MM_F16;
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct ElemTraits<__nv_bfloat16> {
  static constexpr int kCode = B200MM_BF16;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <typename T> __device__ __forceinline__ float to_f(T v) { return ElemTraits<T>::to_f(v); }
template <typename T> __device__ __forceinline__ T from_f(float v) { return ElemTraits<T>::from_f(v); }
template <> __device__ __forceinline__ float to_f<int8_t>(int8_t v) { return (float)v; }

// Unpack one 16-byte chunk of weights into floats.
//   float : 4 elements, half/bf16 : 8 elements, int8 : 16 elements.
template <typename T> struct Chunk;
template <> struct Chunk<float> {
  static constexpr int kElems = 4;
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  }
};
template <> struct Chunk<__nv_bfloat16> {
  static constexpr int kElems = 8;
  // bf16 -> f32 is a 16-bit left shift of the bit pattern.
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <> struct Chunk<__half> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};
template <> struct Chunk<int8_t> {
  static constexpr int kElems = 16;
  // Exact int8 -> f32: flip the sign bit so the byte is u = q + 128 in
  // [1, 255], splice it under the exponent of 2^23 (0x4B000000 | u is the
  // float 2^23 + u), and subtract 2^23 + 128.
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u,
                           v.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // result bytes (LSB first): [byte i of w, 0x00, 0x00, 0x4B]
      f[4 * i + 0] = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7540u)) - 8388736.0f;
      f[4 * i + 1] = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7541u)) - 8388736.0f;
      f[4 * i + 2] = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7542u)) - 8388736.0f;
      f[4 * i + 3] = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7543u)) - 8388736.0f;
    }
  }
};

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

__device__ __forceinline__ float silu_mul(float g, float u) {
  return g / (1.0f + expf(-g)) * u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace b200mm
