// Production-shape MLA split kernel (placeholder: declines every call).
#include "mla.cuh"

namespace b200mm {
bool mla_fast_supported(const MlaDecodeArgs&) { return false; }
int mla_fast_split_launch(const MlaDecodeArgs&, const MlaWorkspace&) { return B200MM_ERR_SHAPE; }
}  // namespace b200mm
