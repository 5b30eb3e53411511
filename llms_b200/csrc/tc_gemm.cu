// Large-M projection kernel on tcgen05 tensor cores (placeholder: declines
// every call until the tensor-core path lands).
#include "dense.cuh"

namespace b200mm {
bool tc_supported(const DenseArgs&) { return false; }
int tc_launch(const DenseArgs&) { return B200MM_ERR_SHAPE; }
}  // namespace b200mm
