/* A plain C caller of libb200mm.so: includes only include/b200mm.h, links the
 * library, and exercises the calls that need no GPU (version, status strings,
 * workspace sizes, argument validation).  Exit status 0 when every check
 * holds; the failing check is printed otherwise. */
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "b200mm.h"

static int failures = 0;
#define CHECK(cond)                                              \
  do {                                                           \
    if (!(cond)) {                                               \
      fprintf(stderr, "abi_check: failed: %s (line %d)\n", #cond, __LINE__); \
      ++failures;                                                \
    }                                                            \
  } while (0)

int main(void) {
  CHECK(b200mm_abi_version() == B200MM_ABI_VERSION);
  CHECK(strcmp(b200mm_status_string(B200MM_OK), "ok") == 0);
  CHECK(strcmp(b200mm_status_string(12345), "unknown status") == 0);

  const uint64_t before = b200mm_launch_count();
  void* p = (void*)(uintptr_t)4096; /* never dereferenced: every call below fails validation */
  CHECK(b200mm_gate_up_silu(NULL, 64, p, 64, p, 64, p, 64, 1, 64, 64, B200MM_BF16, NULL) == B200MM_ERR_ARG);
  CHECK(b200mm_qkv(p, 64, p, 64, p, 96, 1, 96, 0, B200MM_BF16, NULL) == B200MM_ERR_SHAPE);
  CHECK(b200mm_linear(p, 64, p, 64, p, 32, 1, 32, 64, 42, NULL) == B200MM_ERR_DTYPE);
  CHECK(b200mm_linear(p, 64, p, 64, p, 32, 0, 32, 64, B200MM_BF16, NULL) == B200MM_OK); /* M == 0 */

  /* peer output: layout (mirrored by llms_b200._capi.PeerOut) and validation */
  CHECK(sizeof(b200mm_peer_out) == 200);
  CHECK(offsetof(b200mm_peer_out, ld_dst) == 64 && offsetof(b200mm_peer_out, nparts) == 96);
  CHECK(offsetof(b200mm_peer_out, flags) == 112 && offsetof(b200mm_peer_out, err) == 192);
  CHECK(b200mm_linear_peer(p, 64, p, 64, 1, 32, 64, B200MM_BF16, NULL, NULL) == B200MM_ERR_ARG);
  b200mm_peer_out po;
  memset(&po, 0, sizeof(po));
  CHECK(b200mm_linear_peer(p, 64, p, 64, 1, 32, 64, B200MM_BF16, &po, NULL) == B200MM_ERR_ARG); /* world 0 */
  po.world = 2; po.rank = 0; po.nparts = 1; po.part_widths[0] = 16; po.ld_dst = 64;
  po.dst[0] = po.dst[1] = p; po.flags[0] = po.flags[1] = p; po.ticket = po.seen = po.err = p;
  CHECK(b200mm_linear_peer(p, 64, p, 64, 1, 32, 64, B200MM_BF16, &po, NULL) == B200MM_ERR_SHAPE); /* 16 != N */
  CHECK(b200mm_gate_up_silu_w8_peer(p, 64, p, p, p, p, 64, 0, 16, 64, B200MM_BF16, &po, NULL) == B200MM_OK);
  {
    int64_t w = 16;
    void* ptrs[2] = {p, p};
    CHECK(b200mm_peer_gather(p, 16, 1, &w, 1, ptrs, 32, 42, 0, 2, ptrs, p, p, 16, NULL) == B200MM_ERR_DTYPE);
  }

  b200mm_mla_shape s = {1, 32, 8, 128, 32, 256, B200MM_BF16, 1e-6f};
  CHECK(b200mm_mla_decode_workspace_size(&s, 32768) > 0);
  s.DR = 33; /* odd rope width */
  CHECK(b200mm_mla_decode_workspace_size(&s, 32768) == 0);

  const size_t gws = b200mm_gqa_decode_workspace_size(32, 32, 8, 128, 32768);
  CHECK(gws > 0 && gws % 256 == 0);
  CHECK(b200mm_gqa_decode_workspace_size(32, 32, 7, 128, 32768) == 0);
  CHECK(b200mm_gqa_decode(p, 4096, 128, p, 1 << 20, 1 << 17, 128, p, 1 << 20, 1 << 17, 128, p, 4096, 128,
                          32, 32, 8, 128, 1024, 0.088f, B200MM_BF16, p, 16, NULL) == B200MM_ERR_WORKSPACE);

  CHECK(b200mm_launch_count() == before);
  if (failures == 0) printf("abi_check: ok\n");
  return failures ? 1 : 0;
}
