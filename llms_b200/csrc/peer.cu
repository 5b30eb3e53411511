// Column-block all-gather over peer memory (NVLink), for the column-sharded
// decode step: every rank holds the output columns of its shard of a
// projection, y [rows, c], and every rank needs the full [rows, world * c].
//
// One launch per gather, no library collective: each CTA copies its share of
// the local block straight into every rank's gathered buffer (plain 16-byte
// stores through the peers' mapped addresses), at the block's final column
// position -- for a projection with parts (the fused QKV: q | k | v) each part
// lands in its own column range, [q_0 .. q_{n-1} | k_0 .. | v_0 ..], so the
// gathered buffer is the full-width output with no permute afterwards.  Then
// the CTA raises its flag on every peer (a release add at system scope) and
// waits, bounded, until every peer's CTA of the same index has raised its
// flag here: when the kernel ends, every rank's block has arrived.
//
// Flags are monotonic counters: flags[src][cta] on rank r counts the gathers
// in which rank src's CTA `cta` finished writing into rank r; seen[cta]
// (local) counts the gathers this rank's CTA `cta` has completed.  All ranks
// issue the same sequence of gathers, so a CTA waits for flags >= seen + 1.
// A wait that runs out sets *err and the CTA returns (its data may then be
// incomplete; callers check the status word).
#include "common.cuh"
#include "tma.cuh"

namespace b200mm {

namespace {

constexpr int kPeerMax = 8;
constexpr int kThreads = 256;
constexpr unsigned long long kPeerWaitNs = 5ull * 1000 * 1000 * 1000;  // 5 s

struct PeerGatherParams {
  const char* src;
  int64_t ld_src;  // bytes
  int64_t rows;
  int nparts;
  int64_t wbytes[3];    // width of part j in this rank's block, bytes
  int64_t src_off[3];   // column offset of part j in the local block, bytes
  int64_t dst_off[3];   // column offset of part j's rank-0 block in the gathered row, bytes
  int64_t ld_dst;       // bytes
  char* dst[kPeerMax];  // every rank's gathered buffer (this rank's own included)
  unsigned* flags[kPeerMax];  // every rank's flag array [world][kPeerCtas]
  unsigned* seen;       // local [kPeerCtas]
  int* err;             // local status word
  int rank, world, vec; // vec: bytes per copy (16, 8, 4 or 2)
};

__device__ __forceinline__ void red_release_sys(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <int V>
__device__ __forceinline__ void copy_parts(const PeerGatherParams& p) {
  using Vec = typename std::conditional<V == 16, uint4,
              typename std::conditional<V == 8, uint2,
              typename std::conditional<V == 4, uint32_t, uint16_t>::type>::type>::type;
  int64_t per_row = 0;
  for (int j = 0; j < p.nparts; ++j) per_row += p.wbytes[j] / V;
  const int64_t total = per_row * p.rows;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / per_row;
    int64_t col = (i - row * per_row) * V;  // byte offset within the row's block
    int j = 0;
    while (j + 1 < p.nparts && col >= p.wbytes[j]) col -= p.wbytes[j++];
    const Vec v = *reinterpret_cast<const Vec*>(p.src + row * p.ld_src + p.src_off[j] + col);
    const int64_t d = row * p.ld_dst + p.dst_off[j] + (int64_t)p.rank * p.wbytes[j] + col;
    for (int r = 0; r < p.world; ++r) *reinterpret_cast<Vec*>(p.dst[r] + d) = v;
  }
}

__global__ void __launch_bounds__(kThreads) peer_gather_kernel(const PeerGatherParams p) {
  const unsigned expect = p.seen[blockIdx.x] + 1u;
  switch (p.vec) {
    case 16: copy_parts<16>(p); break;
    case 8: copy_parts<8>(p); break;
    case 4: copy_parts<4>(p); break;
    default: copy_parts<2>(p); break;
  }
  __syncthreads();  // the CTA's stores are issued and visible to its threads
  const int t = threadIdx.x;
  // the barrier orders the CTA's stores before thread t's release add, and a
  // release is cumulative: a peer that acquires the count sees every store
  // (no full system fence: it cost ~3.4 us per gather, measured)
  if (t < p.world && t != p.rank) red_release_sys(p.flags[t] + (size_t)p.rank * gridDim.x + blockIdx.x, 1u);
  if (t < p.world && t != p.rank) {
    const unsigned* f = p.flags[p.rank] + (size_t)t * gridDim.x + blockIdx.x;
    const unsigned long long t0 = global_ns();
    while ((int)(ld_acquire_sys(f) - expect) < 0) {
      if (global_ns() - t0 > kPeerWaitNs) {
        atomicExch(p.err, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (t == 0) p.seen[blockIdx.x] = expect;
}

}  // namespace

int peer_gather_launch(const void* src, int64_t ld_src, int64_t rows, const int64_t* widths, int nparts,
                       void* const* dst, int64_t ld_dst, int elem_bytes, int rank, int world, unsigned* const* flags,
                       unsigned* seen, int* err, int nctas, cudaStream_t stream) {
  if (!src || !widths || !dst || !flags || !seen || !err) return B200MM_ERR_ARG;
  if (world < 1 || world > kPeerMax || rank < 0 || rank >= world) return B200MM_ERR_ARG;
  if (nparts < 1 || nparts > 3 || rows < 0 || nctas < 1 || nctas > 1024) return B200MM_ERR_SHAPE;
  if (elem_bytes != 2 && elem_bytes != 4) return B200MM_ERR_DTYPE;
  PeerGatherParams p = {};
  p.src = static_cast<const char*>(src);
  p.ld_src = ld_src * elem_bytes;
  p.ld_dst = ld_dst * elem_bytes;
  p.rows = rows;
  p.nparts = nparts;
  int64_t so = 0, full = 0;
  for (int j = 0; j < nparts; ++j) {
    if (widths[j] <= 0) return B200MM_ERR_SHAPE;
    p.wbytes[j] = widths[j] * elem_bytes;
    p.src_off[j] = so;
    p.dst_off[j] = full;
    so += p.wbytes[j];
    full += p.wbytes[j] * world;
  }
  if (so > p.ld_src || full > p.ld_dst) return B200MM_ERR_SHAPE;
  // the widest copy every address, width and stride allows
  uint64_t bits = (uint64_t)p.ld_src | (uint64_t)p.ld_dst | (uintptr_t)src;
  for (int j = 0; j < nparts; ++j) bits |= (uint64_t)p.wbytes[j];
  for (int r = 0; r < world; ++r) {
    if (!dst[r] || !flags[r]) return B200MM_ERR_ARG;
    bits |= (uintptr_t)dst[r];
    p.dst[r] = static_cast<char*>(dst[r]);
    p.flags[r] = flags[r];
  }
  if ((uintptr_t)seen % 4 || (uintptr_t)err % 4) return B200MM_ERR_ALIGN;
  p.vec = (bits & 15) == 0 ? 16 : (bits & 7) == 0 ? 8 : (bits & 3) == 0 ? 4 : 2;
  if (bits & 1) return B200MM_ERR_ALIGN;
  p.seen = seen;
  p.err = err;
  p.rank = rank;
  p.world = world;
  if (rows == 0) return B200MM_OK;
  count_launch();
  peer_gather_kernel<<<nctas, kThreads, 0, stream>>>(p);
  return launch_status();
}

}  // namespace b200mm
