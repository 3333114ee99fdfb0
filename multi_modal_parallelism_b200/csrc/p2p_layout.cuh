// Layout of a rank's peer-memory all-reduce buffer, shared by the all-reduce kernel (p2p.cu) and the decode GEMM
// that writes its output tiles straight into every rank's buffer (gemm_tc.cu):
//   slots     [2 parity][world source][rows_max][H] bf16   (call e uses parity e & 1)
//   flags     [rows_max][world] u32                         (epoch of the last push of a row, per source)
//   epoch, done                 u32, u32                    (calls completed on this rank; CTA counter)
//   counters  [world] u64                                   (elements the GEMM path received from each source)
//   target    u64                                           (elements expected from each source so far)
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace mmp {

struct PeerBufs {
  const uint64_t* bufs;  // [world] base address of every rank's buffer in this process; null = no peer push
  int rank, world, rows_max, H;
};

__host__ __device__ inline size_t ar_slots_bytes(int world, int rows_max, int H) {
  return 2ull * world * rows_max * H * 2;
}
__host__ __device__ inline size_t ar_flags_off(int world, int rows_max, int H) { return ar_slots_bytes(world, rows_max, H); }
__host__ __device__ inline size_t ar_epoch_off(int world, int rows_max, int H) {
  return ar_flags_off(world, rows_max, H) + static_cast<size_t>(rows_max) * world * 4;
}
__host__ __device__ inline size_t ar_counters_off(int world, int rows_max, int H) {
  return (ar_epoch_off(world, rows_max, H) + 8 + 7) / 8 * 8;
}
__host__ __device__ inline size_t ar_target_off(int world, int rows_max, int H) {
  return ar_counters_off(world, rows_max, H) + static_cast<size_t>(world) * 8;
}
__host__ __device__ inline size_t ar_total_bytes(int world, int rows_max, int H) {
  return (ar_target_off(world, rows_max, H) + 8 + 15) / 16 * 16;
}

// Element (row, col) of source `src`'s slot, parity `par`, in the buffer at `base`
__host__ __device__ inline uint64_t ar_slot_elem(uint64_t base, const PeerBufs& B, int par, int src, int row, int col) {
  return base + ((static_cast<uint64_t>(par) * B.world + src) * B.rows_max + row) * static_cast<uint64_t>(B.H) * 2 +
         static_cast<uint64_t>(col) * 2;
}

}  // namespace mmp
