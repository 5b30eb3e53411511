// b200mm_mla_decode_noalloc: the MLA decode step for callers that cannot
// allocate device memory.
//
// Some hosts of this library may not call cudaMalloc (or any allocator) at
// decode time: an inference server that hands out memory from a fixed arena
// it reserved up front, a CUDA-graph replay path whose node set must not
// change, or a plugin whose host framework owns every allocation.  They can
// pass inputs and outputs, but not the split-K workspace b200mm_mla_decode
// needs.  This entry point runs the same kernels with that workspace taken
// from a fixed array compiled into the library (g_mla_scratch below, 8 MiB).
// Every GPU that loads the library holds that array until the process exits.
#include <mutex>

#include "mla.cuh"

namespace b200mm {
namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;  // 8 MiB: B = 32, L = 32768 needs ~7.8 MiB
__device__ __align__(256) unsigned char g_mla_scratch[kScratchBytes];

constexpr int kMaxDev = 64;
void* g_scratch_addr[kMaxDev] = {nullptr};
std::mutex g_scratch_mu;

// Device address of g_mla_scratch on the current device, looked up once per
// device.  In host code the array's name is only a host-side handle, never a
// device address, so the kernels get this looked-up pointer instead.
int scratch_address(void** out) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDev) return B200MM_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_mla_scratch) != cudaSuccess || !p) {
      cudaGetLastError();  // do not leave the lookup failure for the next launch check
      return B200MM_ERR_DEVICE;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return B200MM_OK;
}

}  // namespace
}  // namespace b200mm

extern "C" int b200mm_mla_decode_noalloc(const b200mm_mla_shape* shape, const void* q, int64_t q_sb,
                                         const void* c_kv, int64_t c_sb, int64_t c_st, const void* kz,
                                         int64_t z_sb, int64_t z_st, const float* kscale, int64_t s_sb,
                                         int64_t s_st, const void* w_uk, const void* w_uv, const float* k_norm_w,
                                         const float* rope_inv_freq, float scale, int64_t L, void* out,
                                         int64_t o_sb, void* stream) {
  using namespace b200mm;
  if (!shape) return B200MM_ERR_ARG;
  const int st = mla_validate_shape(*shape);
  if (st != B200MM_OK) return st;
  if (L < 1 || L >= (int64_t(1) << 31)) return B200MM_ERR_SHAPE;
  if (shape->B == 0) return B200MM_OK;
  // the workspace this call needs must fit in the fixed array
  if (mla_workspace_bytes(*shape, L) > kScratchBytes) return B200MM_ERR_WORKSPACE;
  void* ws = nullptr;
  const int sa = scratch_address(&ws);
  if (sa != B200MM_OK) return sa;
  // Same kernels as b200mm_mla_decode.  They write every workspace byte they
  // read (the absorbed query, the partials and the error flag) before reading
  // it, so the array's contents from the previous call need no clearing.
  return b200mm_mla_decode(shape, q, q_sb, c_kv, c_sb, c_st, kz, z_sb, z_st, kscale, s_sb, s_st, w_uk, w_uv,
                           k_norm_w, rope_inv_freq, scale, L, out, o_sb, ws, kScratchBytes, stream);
}
