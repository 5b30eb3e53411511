// MLA latent decode, production shape (R=256, D=128, DR=32, H=32, KV=8;
// bf16 or fp16): when the tensor-core split kernel applies, and its TMA
// tensor maps (the token extent is L,
// so rows past the context arrive as zeros).
#include "mla.cuh"

namespace b200mm {

namespace {

constexpr int FR = 256, FD = 128, FDR = 32, FH = 32, FKV = 8;
constexpr int TT = kMlaUnit;  // 64 tokens per unit

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
  // c and kz as [batch][4 column blocks][token][64]: one TMA instruction brings
  // a unit's four 64-column boxes, landing as four consecutive swizzled boxes
  const uint64_t cd[4] = {64, L, 4, B}, zd[4] = {64, L, 4, B};
  const uint64_t cs[3] = {(uint64_t)a.c_st * 2, 128, csb}, zs[3] = {(uint64_t)a.z_st * 2, 128, zsb};
  const uint32_t box[4] = {64, (uint32_t)TT, 4, 1};
  return make_map_4d(&m->c, dt, a.c_kv, cd, cs, box, CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_map_4d(&m->kz, dt, a.kz, zd, zs, box, CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_map_3d(&m->ks, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.kscale, FKV, L, B, (uint64_t)a.s_st * 4, ssb, FKV,
                     TT, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace b200mm
