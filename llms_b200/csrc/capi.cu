// extern "C" entry points of libb200mm.so: argument validation on the host,
// then dispatch to the kernel families.  Declarations and the reference
// interfaces they replace are in include/b200mm.h.
#include <mutex>

#include "dense.cuh"

#include <cstdlib>
#include <string>
#include "mla.cuh"

namespace b200mm {

std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_force_generic{0};

namespace {
constexpr int kMaxDev = 64;
int g_sms[kMaxDev] = {0};
int g_cc_ok[kMaxDev] = {0};  // 0 unknown, 1 sm_100, -1 other
}  // namespace

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

int num_sms(int device) {
  if (device < 0 || device >= kMaxDev) return 148;
  if (g_sms[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
    g_sms[device] = v;
  }
  return g_sms[device];
}

// The kernels are compiled for sm_100a only; refuse other devices up front
// instead of failing with "no kernel image" at launch.
int check_device() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDev) return B200MM_ERR_DEVICE;
  if (g_cc_ok[d] == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d) != cudaSuccess)
      return B200MM_ERR_DEVICE;
    g_cc_ok[d] = (major == 10 && minor == 0) ? 1 : -1;
  }
  return g_cc_ok[d] == 1 ? B200MM_OK : B200MM_ERR_DEVICE;
}

int dense_dispatch(const DenseArgs& a) {
  // peer output: the decode-regime families that carry the gather epilogue,
  // chosen exactly as below
  if (a.peer) {
    if (a.M <= (a.w8 ? 1 : 4) && gemv_supported(a)) return gemv_launch(a);
    if (a.M <= (a.w8 ? 32 : a.gate ? 16 : 8) && mmv_supported(a)) return mmv_launch(a);
    return B200MM_ERR_SHAPE;
  }
  if (g_force_generic.load(std::memory_order_relaxed)) return tiled_launch(a);
#ifdef SWAP_TRACE
  // development builds only: force one family ("gemv", "mmv", "swap", "tc")
  if (const char* f = getenv("B200MM_DENSE_FAMILY")) {
    const std::string fam(f);
    if (fam == "gemv" && gemv_supported(a)) return gemv_launch(a);
    if (fam == "mmv" && mmv_supported(a)) return mmv_launch(a);
    if (fam == "swap" && swap_supported(a)) return swap_launch(a);
    if (fam == "tc" && tc_supported(a)) return tc_launch(a);
  }
#endif
  // measured on B200 at the Qwen3 shapes: M <= 4 CUDA-core GEMV (int8: M = 1;
  // at M = 2..4 the mma.sync GEMV took 10 us for the 8B int8 QKV where the
  // CUDA-core GEMV took 16); small M the mma.sync GEMV (gate-up M <= 16,
  // plain projections M <= 8, int8 M <= 32);
  // then tcgen05 with the weights as the MMA's M side (16-bit up to M = 64,
  // and up to 128 for narrow plain projections (FFN down, K >= 2N, and
  // outputs up to 3072 wide such as the 2560-wide o), whose few output tiles
  // leave the GEMM tiled over X short of CTAs; int8 any M); otherwise the
  // tcgen05 GEMM tiled over X
  const bool narrow_deep = !a.gate && (a.K >= 2 * a.N || a.N <= 3072);
  if (a.M <= (a.w8 ? 1 : 4) && gemv_supported(a)) return gemv_launch(a);
  if (a.M <= (a.w8 ? 32 : a.gate ? 16 : 8) && mmv_supported(a)) return mmv_launch(a);
  if ((a.w8 || a.M <= 64 || (narrow_deep && a.M <= 128)) && swap_supported(a)) return swap_launch(a);
  if (tc_supported(a)) return tc_launch(a);
  if (mmv_supported(a)) return mmv_launch(a);
  if (gemv_supported(a)) return gemv_launch(a);
  return tiled_launch(a);
}

namespace {

int validate_dense(const DenseArgs& a) {
  if (!a.x || !a.w0 || !a.y || (a.gate && !a.w1)) return B200MM_ERR_ARG;
  if (a.w8 && (!a.s0 || (a.gate && !a.s1))) return B200MM_ERR_ARG;
  if (a.dtype != B200MM_F32 && a.dtype != B200MM_F16 && a.dtype != B200MM_BF16) return B200MM_ERR_DTYPE;
  if (a.w8 && a.dtype == B200MM_F32) return B200MM_ERR_DTYPE;
  if (a.M < 0 || a.N < 1 || a.K < 1) return B200MM_ERR_SHAPE;
  if (a.ldx < a.K || a.ldw0 < a.K || (a.gate && a.ldw1 < a.K) || a.ldy < a.N) return B200MM_ERR_SHAPE;
  return B200MM_OK;
}

bool fits_i32(int64_t v) { return v >= 0 && v < (int64_t(1) << 31); }

int validate_peer(const b200mm_peer_out& po, int64_t N) {
  if (po.world < 1 || po.world > 8 || po.rank < 0 || po.rank >= po.world) return B200MM_ERR_ARG;
  if (po.nparts < 1 || po.nparts > 3) return B200MM_ERR_SHAPE;
  int64_t sum = 0;
  for (int j = 0; j < po.nparts; ++j) {
    if (po.part_widths[j] < 1) return B200MM_ERR_SHAPE;
    sum += po.part_widths[j];
  }
  if (sum != N || po.ld_dst < sum * po.world) return B200MM_ERR_SHAPE;
  for (int r = 0; r < po.world; ++r)
    if (!po.dst[r] || !po.flags[r] || ((uintptr_t)po.flags[r] & 3u)) return B200MM_ERR_ARG;
  if (!po.ticket || !po.seen || !po.err) return B200MM_ERR_ARG;
  return B200MM_OK;
}

int run_dense(DenseArgs& a, int64_t M, int64_t N, int64_t K) {
  if (!fits_i32(M) || !fits_i32(N) || !fits_i32(K)) return B200MM_ERR_SHAPE;
  a.M = (int)M; a.N = (int)N; a.K = (int)K;
  if (a.peer) {
    const int st = validate_peer(*a.peer, N);
    if (st != B200MM_OK) return st;
    a.y = a.peer->dst[a.peer->rank];  // (unused: the epilogue stores through dst[])
    a.ldy = a.peer->ld_dst;
  }
  int st = validate_dense(a);
  if (st != B200MM_OK) return st;
  if (a.M == 0) return B200MM_OK;
  st = check_device();
  if (st != B200MM_OK) return st;
  st = dense_dispatch(a);
  if (st != B200MM_OK) return st;
  return launch_status();
}

}  // namespace
}  // namespace b200mm

using namespace b200mm;

extern "C" {

const char* b200mm_status_string(int s) {
  switch (s) {
    case B200MM_OK: return "ok";
    case B200MM_ERR_SHAPE: return "invalid or unsupported shape";
    case B200MM_ERR_ALIGN: return "pointer or stride alignment not supported";
    case B200MM_ERR_DTYPE: return "unsupported dtype";
    case B200MM_ERR_LAUNCH: return "kernel launch failed";
    case B200MM_ERR_ARG: return "null pointer or invalid argument";
    case B200MM_ERR_WORKSPACE: return "workspace missing or too small";
    case B200MM_ERR_DEVICE: return "device is not an sm_100 GPU or a device query failed";
    case B200MM_ERR_TIMEOUT: return "an on-device wait timed out";
    default: return "unknown status";
  }
}

int b200mm_abi_version(void) { return B200MM_ABI_VERSION; }

uint64_t b200mm_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int b200mm_force_generic(int on) { return g_force_generic.exchange(on ? 1 : 0); }

int b200mm_gate_up_silu(const void* x, int64_t ldx, const void* wg, int64_t ldwg, const void* wu,
                        int64_t ldwu, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                        int dtype, void* stream) {
  DenseArgs a{};
  a.x = x; a.ldx = ldx; a.w0 = wg; a.ldw0 = ldwg; a.w1 = wu; a.ldw1 = ldwu;
  a.y = y; a.ldy = ldy; a.dtype = dtype; a.w8 = false; a.gate = true;
  a.stream = static_cast<cudaStream_t>(stream);
  return run_dense(a, M, N, K);
}

int b200mm_qkv(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
               int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  DenseArgs a{};
  a.x = x; a.ldx = ldx; a.w0 = w; a.ldw0 = ldw; a.y = y; a.ldy = ldy;
  a.dtype = dtype; a.w8 = false; a.gate = false;
  a.stream = static_cast<cudaStream_t>(stream);
  return run_dense(a, M, N, K);
}

int b200mm_gate_up_silu_w8(const void* x, int64_t ldx, const int8_t* wg, const float* sg,
                           const int8_t* wu, const float* su, int64_t ldw, void* y, int64_t ldy,
                           int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  DenseArgs a{};
  a.x = x; a.ldx = ldx; a.w0 = wg; a.ldw0 = ldw; a.w1 = wu; a.ldw1 = ldw;
  a.s0 = sg; a.s1 = su; a.y = y; a.ldy = ldy; a.dtype = dtype; a.w8 = true; a.gate = true;
  a.stream = static_cast<cudaStream_t>(stream);
  return run_dense(a, M, N, K);
}

int b200mm_qkv_w8(const void* x, int64_t ldx, const int8_t* w, const float* s, int64_t ldw,
                  void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  DenseArgs a{};
  a.x = x; a.ldx = ldx; a.w0 = w; a.ldw0 = ldw; a.s0 = s; a.y = y; a.ldy = ldy;
  a.dtype = dtype; a.w8 = true; a.gate = false;
  a.stream = static_cast<cudaStream_t>(stream);
  return run_dense(a, M, N, K);
}

int b200mm_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                  int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  return b200mm_qkv(x, ldx, w, ldw, y, ldy, M, N, K, dtype, stream);
}

int b200mm_linear_w8(const void* x, int64_t ldx, const int8_t* w, const float* s, int64_t ldw,
                     void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  return b200mm_qkv_w8(x, ldx, w, s, ldw, y, ldy, M, N, K, dtype, stream);
}

int b200mm_linear_peer(const void* x, int64_t ldx, const void* w, int64_t ldw, int64_t M, int64_t N, int64_t K,
                       int dtype, const b200mm_peer_out* out, void* stream) {
  if (!out) return B200MM_ERR_ARG;
  DenseArgs a{};
  a.x = x; a.ldx = ldx; a.w0 = w; a.ldw0 = ldw;
  a.dtype = dtype; a.w8 = false; a.gate = false; a.peer = out;
  a.stream = static_cast<cudaStream_t>(stream);
  return run_dense(a, M, N, K);
}

int b200mm_linear_w8_peer(const void* x, int64_t ldx, const int8_t* w, const float* s, int64_t ldw, int64_t M,
                          int64_t N, int64_t K, int dtype, const b200mm_peer_out* out, void* stream) {
  if (!out) return B200MM_ERR_ARG;
  DenseArgs a{};
  a.x = x; a.ldx = ldx; a.w0 = w; a.ldw0 = ldw; a.s0 = s;
  a.dtype = dtype; a.w8 = true; a.gate = false; a.peer = out;
  a.stream = static_cast<cudaStream_t>(stream);
  return run_dense(a, M, N, K);
}

int b200mm_gate_up_silu_w8_peer(const void* x, int64_t ldx, const int8_t* wg, const float* sg, const int8_t* wu,
                                const float* su, int64_t ldw, int64_t M, int64_t N, int64_t K, int dtype,
                                const b200mm_peer_out* out, void* stream) {
  if (!out) return B200MM_ERR_ARG;
  DenseArgs a{};
  a.x = x; a.ldx = ldx; a.w0 = wg; a.ldw0 = ldw; a.w1 = wu; a.ldw1 = ldw;
  a.s0 = sg; a.s1 = su; a.dtype = dtype; a.w8 = true; a.gate = true; a.peer = out;
  a.stream = static_cast<cudaStream_t>(stream);
  return run_dense(a, M, N, K);
}

int b200mm_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, void* h_out, int64_t ldh,
                   const void* weight, void* y, int64_t ldy, int64_t M, int64_t N, float eps, int dtype,
                   void* stream) {
  if (dtype != B200MM_F32 && dtype != B200MM_F16 && dtype != B200MM_BF16) return B200MM_ERR_DTYPE;
  if (M < 0 || M > 2147483647LL || N < 1 || N > 16384) return B200MM_ERR_SHAPE;
  if (ldx < N || ldy < N || (residual && ldr < N) || (h_out && ldh < N)) return B200MM_ERR_SHAPE;
  if (!x || !weight || !y || (h_out && !residual) || !(eps >= 0.f)) return B200MM_ERR_ARG;
  if (M == 0) return B200MM_OK;
  int st = check_device();
  if (st != B200MM_OK) return st;
  st = glue_rmsnorm(x, ldx, residual, ldr, h_out, ldh, weight, y, ldy, (int)M, (int)N, eps, dtype,
                    static_cast<cudaStream_t>(stream));
  if (st != B200MM_OK) return st;
  return launch_status();
}

int b200mm_qk_norm_rope(const void* qkv, int64_t ldq, int64_t B, int64_t H, int64_t KV, int64_t D,
                        const void* q_norm_w, const void* k_norm_w, const void* cos_table, const void* sin_table,
                        int64_t max_pos, int64_t pos, const int64_t* pos_dev, void* q_out, int64_t q_sb,
                        int64_t q_sh, void* k_cache, int64_t k_sb, int64_t k_sh, int64_t k_st, void* v_cache,
                        int64_t v_sb, int64_t v_sh, int64_t v_st, float eps, int dtype, void* stream) {
  if (dtype != B200MM_F32 && dtype != B200MM_F16 && dtype != B200MM_BF16) return B200MM_ERR_DTYPE;
  if (B < 0 || B > 65535 || KV < 1 || H < KV || H % KV || H > 4096 || (D != 64 && D != 128 && D != 256))
    return B200MM_ERR_SHAPE;
  if (ldq < (H + 2 * KV) * D || q_sh < D || q_sb < 0 || k_st < D || v_st < D || k_sh < 0 || v_sh < 0 ||
      k_sb < 0 || v_sb < 0)
    return B200MM_ERR_SHAPE;
  if (!qkv || !q_norm_w || !k_norm_w || !cos_table || !sin_table || !q_out || !k_cache || !v_cache ||
      !(eps >= 0.f))
    return B200MM_ERR_ARG;
  // a host position is checked here; a device position is the caller's to keep in [0, max_pos)
  if (!pos_dev && (pos < 0 || pos >= max_pos)) return B200MM_ERR_SHAPE;
  if (B == 0) return B200MM_OK;
  int st = check_device();
  if (st != B200MM_OK) return st;
  st = glue_qk_norm_rope(qkv, ldq, (int)B, (int)H, (int)KV, (int)D, q_norm_w, k_norm_w, cos_table, sin_table, pos,
                         pos_dev, q_out, q_sb, q_sh, k_cache, k_sb, k_sh, k_st, v_cache, v_sb, v_sh, v_st, eps, dtype,
                         static_cast<cudaStream_t>(stream));
  if (st != B200MM_OK) return st;
  return launch_status();
}

namespace {
bool gqa_shape_ok(int64_t B, int64_t H, int64_t KV, int64_t D, int64_t L) {
  return B >= 0 && B <= 65535 && KV >= 1 && H >= KV && H <= 65535 && H % KV == 0 && D >= 2 && D <= 1024 &&
         D % 2 == 0 && L >= 1 && L < (int64_t(1) << 31);
}
}  // namespace

size_t b200mm_gqa_decode_workspace_size(int64_t B, int64_t H, int64_t KV, int64_t D, int64_t L) {
  if (!gqa_shape_ok(B, H, KV, D, L)) return 0;
  return gqa_workspace_bytes((int)(B > 0 ? B : 1), (int)H, (int)KV, (int)D, L);
}

int b200mm_gqa_decode(const void* q, int64_t q_sb, int64_t q_sh, const void* k, int64_t k_sb, int64_t k_sh,
                      int64_t k_st, const void* v, int64_t v_sb, int64_t v_sh, int64_t v_st, void* out,
                      int64_t o_sb, int64_t o_sh, int64_t B, int64_t H, int64_t KV, int64_t D, int64_t L,
                      float scale, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != B200MM_F32 && dtype != B200MM_F16 && dtype != B200MM_BF16) return B200MM_ERR_DTYPE;
  if (!gqa_shape_ok(B, H, KV, D, L)) return B200MM_ERR_SHAPE;
  if (!q || !k || !v || !out || !(scale > 0.f)) return B200MM_ERR_ARG;
  if (q_sb < 0 || q_sh < 0 || k_sb < 0 || k_sh < 0 || k_st < D || v_sb < 0 || v_sh < 0 || v_st < D || o_sb < 0 ||
      o_sh < 0)
    return B200MM_ERR_SHAPE;
  if (B == 0) return B200MM_OK;
  const size_t need = gqa_workspace_bytes((int)B, (int)H, (int)KV, (int)D, L);
  if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255u)) return B200MM_ERR_WORKSPACE;
  int st = check_device();
  if (st != B200MM_OK) return st;
  st = gqa_decode(q, q_sb, q_sh, k, k_sb, k_sh, k_st, v, v_sb, v_sh, v_st, out, o_sb, o_sh, (int)B, (int)H,
                  (int)KV, (int)D, L, scale, dtype, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
  if (st != B200MM_OK) return st;
  return launch_status();
}

int b200mm_mla_append(const b200mm_mla_shape* shape, const void* c_kv, int64_t c_sb, int64_t c_st,
                      const void* k_rope_pre, int64_t r_sb, int64_t r_st, const void* w_uk, const float* k_norm_w,
                      const float* rope_inv_freq, float* kscale, int64_t s_sb, int64_t s_st, void* kz,
                      int64_t z_sb, int64_t z_st, int64_t t0, int64_t t1, void* stream) {
  if (!shape) return B200MM_ERR_ARG;
  MlaAppendArgs a{};
  a.s = *shape;
  a.c_kv = c_kv; a.c_sb = c_sb; a.c_st = c_st;
  a.kr = k_rope_pre; a.r_sb = r_sb; a.r_st = r_st;
  a.w_uk = w_uk; a.k_norm_w = k_norm_w; a.inv_freq = rope_inv_freq;
  a.kscale = kscale; a.s_sb = s_sb; a.s_st = s_st;
  a.kz = kz; a.z_sb = z_sb; a.z_st = z_st;
  a.t0 = t0; a.t1 = t1; a.stream = static_cast<cudaStream_t>(stream);
  int st = mla_validate_shape(a.s);
  if (st != B200MM_OK) return st;
  if (!c_kv || !kscale || (a.s.D - a.s.DR > 0 && !w_uk)) return B200MM_ERR_ARG;
  if (a.s.DR > 0 && (!k_rope_pre || !kz || !k_norm_w || !rope_inv_freq)) return B200MM_ERR_ARG;
  if (t0 < 0 || t1 < t0 || t1 >= (int64_t(1) << 31)) return B200MM_ERR_SHAPE;
  if (t1 == t0 || a.s.B == 0) return B200MM_OK;
  st = check_device();
  if (st != B200MM_OK) return st;
  st = mla_append_launch(a);
  if (st != B200MM_OK) return st;
  return launch_status();
}

size_t b200mm_mla_decode_workspace_size(const b200mm_mla_shape* shape, int64_t L) {
  if (!shape || mla_validate_shape(*shape) != B200MM_OK || L < 1) return 0;
  return mla_workspace_bytes(*shape, L);
}

int b200mm_mla_decode(const b200mm_mla_shape* shape, const void* q, int64_t q_sb, const void* c_kv,
                      int64_t c_sb, int64_t c_st, const void* kz, int64_t z_sb, int64_t z_st,
                      const float* kscale, int64_t s_sb, int64_t s_st, const void* w_uk,
                      const void* w_uv, const float* k_norm_w, const float* rope_inv_freq,
                      float scale, int64_t L, void* out, int64_t o_sb, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (!shape) return B200MM_ERR_ARG;
  MlaDecodeArgs a{};
  a.s = *shape;
  a.q = q; a.q_sb = q_sb;
  a.c_kv = c_kv; a.c_sb = c_sb; a.c_st = c_st;
  a.kz = kz; a.z_sb = z_sb; a.z_st = z_st;
  a.kscale = kscale; a.s_sb = s_sb; a.s_st = s_st;
  a.w_uk = w_uk; a.w_uv = w_uv; a.k_norm_w = k_norm_w; a.inv_freq = rope_inv_freq;
  a.scale = scale; a.L = L; a.out = out; a.o_sb = o_sb;
  a.ws = workspace; a.ws_bytes = workspace_bytes;
  a.stream = static_cast<cudaStream_t>(stream);
  a.qpos = L - 1;
  int st = mla_validate_shape(a.s);
  if (st != B200MM_OK) return st;
  if (L < 1 || L >= (int64_t(1) << 31)) return B200MM_ERR_SHAPE;
  if (!q || !c_kv || !kscale || !w_uv || !k_norm_w || !out) return B200MM_ERR_ARG;
  if (a.s.DR > 0 && (!kz || !rope_inv_freq)) return B200MM_ERR_ARG;
  if (a.s.D - a.s.DR > 0 && !w_uk) return B200MM_ERR_ARG;
  if (!(scale > 0.f)) return B200MM_ERR_ARG;
  if (a.s.B == 0) return B200MM_OK;
  const size_t need = mla_workspace_bytes(a.s, L);
  if (need > 0 && (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255u)))
    return B200MM_ERR_WORKSPACE;
  st = check_device();
  if (st != B200MM_OK) return st;
  st = mla_decode_launch(a);
  if (st != B200MM_OK) return st;
  return launch_status();
}

int b200mm_mla_decode_partial(const b200mm_mla_shape* shape, const void* q, int64_t q_sb, const void* c_kv,
                              int64_t c_sb, int64_t c_st, const void* kz, int64_t z_sb, int64_t z_st,
                              const float* kscale, int64_t s_sb, int64_t s_st, const void* w_uk,
                              const float* k_norm_w, const float* rope_inv_freq, float scale, int64_t L,
                              int64_t t_begin, int64_t t_end, float* av_out, float* ml_out, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (!shape) return B200MM_ERR_ARG;
  int st = mla_validate_shape(*shape);
  if (st != B200MM_OK) return st;
  if (L < 1 || L >= (int64_t(1) << 31) || t_begin < 0 || t_end <= t_begin || t_end > L) return B200MM_ERR_SHAPE;
  if (!q || !c_kv || !kscale || !k_norm_w || !av_out || !ml_out) return B200MM_ERR_ARG;
  if (shape->DR > 0 && (!kz || !rope_inv_freq)) return B200MM_ERR_ARG;
  if (shape->D - shape->DR > 0 && !w_uk) return B200MM_ERR_ARG;
  if (!(scale > 0.f)) return B200MM_ERR_ARG;
  if (shape->B == 0) return B200MM_OK;
  MlaDecodeArgs a{};
  a.s = *shape;
  const int esz = shape->dtype == B200MM_F32 ? 4 : 2;
  // the range's tokens: every per-token pointer starts at t_begin
  a.q = q; a.q_sb = q_sb;
  a.c_kv = static_cast<const unsigned char*>(c_kv) + t_begin * c_st * esz; a.c_sb = c_sb; a.c_st = c_st;
  a.kz = kz ? static_cast<const unsigned char*>(kz) + t_begin * z_st * esz : nullptr; a.z_sb = z_sb; a.z_st = z_st;
  a.kscale = kscale + t_begin * s_st; a.s_sb = s_sb; a.s_st = s_st;
  a.w_uk = w_uk; a.w_uv = nullptr; a.k_norm_w = k_norm_w; a.inv_freq = rope_inv_freq;
  a.scale = scale; a.L = t_end - t_begin; a.qpos = L - 1;
  a.av_out = av_out; a.ml_out = ml_out;
  a.ws = workspace; a.ws_bytes = workspace_bytes;
  a.stream = static_cast<cudaStream_t>(stream);
  const size_t need = mla_workspace_bytes(a.s, a.L);
  if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255u)) return B200MM_ERR_WORKSPACE;
  st = check_device();
  if (st != B200MM_OK) return st;
  st = mla_decode_launch(a);
  if (st != B200MM_OK) return st;
  return launch_status();
}

int b200mm_mla_combine_partials(const b200mm_mla_shape* shape, const float* av_parts, int64_t av_part_stride,
                                const float* ml_parts, int64_t ml_part_stride, int64_t nparts, const void* w_uv,
                                void* out, int64_t o_sb, void* workspace, size_t workspace_bytes, void* stream) {
  if (!shape) return B200MM_ERR_ARG;
  int st = mla_validate_shape(*shape);
  if (st != B200MM_OK) return st;
  if (nparts < 1 || nparts > 64) return B200MM_ERR_SHAPE;
  if (!av_parts || !ml_parts || !w_uv || !out) return B200MM_ERR_ARG;
  const int64_t bh = (int64_t)shape->B * shape->H;
  if (av_part_stride < bh * shape->R || ml_part_stride < bh * 2) return B200MM_ERR_SHAPE;
  if (shape->B == 0) return B200MM_OK;
  MlaDecodeArgs a{};
  a.s = *shape;
  a.w_uv = w_uv; a.out = out; a.o_sb = o_sb; a.L = 1; a.qpos = 0;
  a.ws = workspace; a.ws_bytes = workspace_bytes;
  a.stream = static_cast<cudaStream_t>(stream);
  const size_t need = mla_workspace_bytes(a.s, 1);
  if (!workspace || workspace_bytes < need || ((uintptr_t)workspace & 255u)) return B200MM_ERR_WORKSPACE;
  st = check_device();
  if (st != B200MM_OK) return st;
  st = mla_combine_partials_launch(a, av_parts, av_part_stride, ml_parts, ml_part_stride, (int)nparts);
  if (st != B200MM_OK) return st;
  return launch_status();
}

int b200mm_peer_gather(const void* src, int64_t ld_src, int64_t rows, const int64_t* part_widths, int nparts,
                       void* const* dst, int64_t ld_dst, int dtype, int rank, int world, void* const* flags,
                       void* seen, void* err, int nctas, void* stream) {
  const int eb = dtype == B200MM_F32 ? 4 : (dtype == B200MM_F16 || dtype == B200MM_BF16) ? 2 : 0;
  if (!eb) return B200MM_ERR_DTYPE;
  int st = check_device();
  if (st != B200MM_OK) return st;
  return peer_gather_launch(src, ld_src, rows, part_widths, nparts, dst, ld_dst, eb, rank, world,
                            reinterpret_cast<unsigned* const*>(flags), static_cast<unsigned*>(seen),
                            static_cast<int*>(err), nctas, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
