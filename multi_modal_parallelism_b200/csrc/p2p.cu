// Peer-memory all-reduce for the layer's [rows, H] partial sums, fused with what follows it in the layer:
// a one-shot all-reduce over NVLink (every rank pushes its partial into every rank's buffer with plain peer
// stores, then sums the world's partials locally in rank order), the residual add and, optionally, the RMSNorm
// of the sum. Replaces the NCCL all-reduce of the reference's `ParallelHybridLayer._ar` (harness/layer.py:175-181)
// and the residual / norm after it (harness/layer.py:217-227) for decode-sized messages, where a collective is
// latency-bound: one launch, no proxy thread, and the reduction lands where the next op needs it.
//
// Buffers: each rank owns one buffer that every rank maps (CUDA IPC): two parity halves of N slots of
// [rows_max, H] bf16 (slot q = rank q's partial), then a flag word per (row, source rank), then an epoch word
// and a done counter. Call e (the epoch, counted on the device) uses parity e & 1, so a rank that runs ahead
// into call e + 1 writes the other half and cannot overwrite partials a slower rank is still summing; flags
// hold the epoch of the last push, so they never need resetting. Each CTA copies its rows of the local partial
// into slot `rank` of every rank's buffer, fences (system scope), raises the rows' flags on every rank (release),
// waits (bounded) until every rank's flags for those rows reach the epoch (acquire), then sums the N slots in
// rank order (every rank computes bit-identical results), adds the residual and normalises. The grid is at most
// one CTA per SM (CTA c owns rows c, c + grid, ...), so all CTAs are resident together.
// Waits give up after a bounded number of polls: the kernel then sets MMP_DEVERR_TIMEOUT and skips the sum.
//
// Fused form (`pushed`): the decode GEMM that produced the partial already wrote its output tiles into slot
// `rank` of every rank's buffer and added the number of elements it wrote to its counter on every rank
// (gemm_tc.cu), so the transfer overlapped the GEMM; this kernel then only waits until every source's counter
// reaches the cumulative target (rows x H per call), sums and normalises.
#include <cuda.h>

#include <map>
#include <mutex>

#include "mmp_common.cuh"
#include "p2p_layout.cuh"

namespace mmp {
namespace {

constexpr int AR_THREADS = 256;
constexpr int AR_MAX_WORLD = 8;
constexpr long long AR_MAX_POLLS = 1LL << 25;  // with 128 ns sleeps: several seconds

struct ArJoinParams {  // element strides
  const uint64_t* bufs;    // [world] base address of every rank's buffer in this process
  int rank, world;
  int rows, H, rows_max;
  int pushed;              // 1: the producing GEMM already pushed the partial (wait on the counters)
  const bf16* part; int64_t p_b;      // local partial [rows, H]
  const bf16* resid; int64_t r_b;     // residual [rows, H] or null
  bf16* sum_out; int64_t s_b;         // residual + all-reduced partials [rows, H]
  const bf16* norm_w; float eps;      // RMSNorm weight [H] or null
  bf16* norm_out; int64_t n_b;        // rmsnorm(sum_out) * w [rows, H]
  int* err;
};

__device__ __forceinline__ uint32_t* flag_ptr(uint64_t base, const ArJoinParams& P, int row, int src) {
  return reinterpret_cast<uint32_t*>(base + ar_flags_off(P.world, P.rows_max, P.H)) + row * P.world + src;
}
__device__ __forceinline__ uint32_t* epoch_ptr(uint64_t base, const ArJoinParams& P) {
  return reinterpret_cast<uint32_t*>(base + ar_epoch_off(P.world, P.rows_max, P.H));
}
__device__ __forceinline__ uint64_t* counter_ptr(uint64_t base, const ArJoinParams& P, int src) {
  return reinterpret_cast<uint64_t*>(base + ar_counters_off(P.world, P.rows_max, P.H)) + src;
}
__device__ __forceinline__ uint64_t* target_ptr(uint64_t base, const ArJoinParams& P) {
  return reinterpret_cast<uint64_t*>(base + ar_target_off(P.world, P.rows_max, P.H));
}
__device__ __forceinline__ uint64_t ld_acquire_sys64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void push_row(const ArJoinParams& P, int row, int par, size_t slot_elems) {
  const uint4* src = reinterpret_cast<const uint4*>(P.part + row * P.p_b);
  for (int v = threadIdx.x; v < P.H / 8; v += AR_THREADS) {
    const uint4 x = src[v];
#pragma unroll 1
    for (int q = 0; q < P.world; ++q) {
      bf16* dst = reinterpret_cast<bf16*>(P.bufs[q]) + (static_cast<size_t>(par) * P.world + P.rank) * slot_elems +
                  static_cast<size_t>(row) * P.H;
      reinterpret_cast<uint4*>(dst)[v] = x;
    }
  }
}

// sum_out[row] = bf16(resid[row] + bf16(sum of the world's slots)); returns this thread's sum of squares of it
__device__ __forceinline__ float reduce_row(const ArJoinParams& P, int row, const bf16* slots0, size_t slot_elems,
                                            bool ok) {
  float ss = 0.f;
  const bf16* slots = slots0 + static_cast<size_t>(row) * P.H;
  for (int v = threadIdx.x; v < P.H / 8; v += AR_THREADS) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (ok) {
#pragma unroll 1
      for (int q = 0; q < P.world; ++q) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(slots + q * slot_elems) + v);
        const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
        acc[0] += a.x; acc[1] += a.y; acc[2] += b.x; acc[3] += b.y;
        acc[4] += c.x; acc[5] += c.y; acc[6] += d.x; acc[7] += d.y;
      }
    }
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = bf2f(f2bf(acc[i]));  // the all-reduced partial, as a bf16 tensor
    if (P.resid) {
      const uint4 r = reinterpret_cast<const uint4*>(P.resid + row * P.r_b)[v];
      const float2 a = unpack_bf16x2(r.x), b = unpack_bf16x2(r.y), c = unpack_bf16x2(r.z), d = unpack_bf16x2(r.w);
      const float rr[8] = {a.x, a.y, b.x, b.y, c.x, c.y, d.x, d.y};
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i] = bf2f(f2bf(rr[i] + s[i]));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(s[i], s[i], ss);
    reinterpret_cast<uint4*>(P.sum_out + row * P.s_b)[v] =
        make_uint4(pack_bf16x2(s[0], s[1]), pack_bf16x2(s[2], s[3]), pack_bf16x2(s[4], s[5]), pack_bf16x2(s[6], s[7]));
  }
  return ss;
}

__device__ __forceinline__ void norm_row(const ArJoinParams& P, int row, float r) {
  for (int v = threadIdx.x; v < P.H / 8; v += AR_THREADS) {
    const uint4 u = reinterpret_cast<const uint4*>(P.sum_out + row * P.s_b)[v];
    const uint4 w = reinterpret_cast<const uint4*>(P.norm_w)[v];
    const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
    const float2 wa = unpack_bf16x2(w.x), wb = unpack_bf16x2(w.y), wc = unpack_bf16x2(w.z), wd = unpack_bf16x2(w.w);
    reinterpret_cast<uint4*>(P.norm_out + row * P.n_b)[v] =
        make_uint4(pack_bf16x2(a.x * r * wa.x, a.y * r * wa.y), pack_bf16x2(b.x * r * wb.x, b.y * r * wb.y),
                   pack_bf16x2(c.x * r * wc.x, c.y * r * wc.y), pack_bf16x2(d.x * r * wd.x, d.y * r * wd.y));
  }
}

// Grid <= the SM count, so every CTA of every rank is resident at once and no wait depends on a CTA that has
// not started; CTA c owns rows c, c + grid, ... on every rank.
__global__ void __launch_bounds__(AR_THREADS) ar_join_kernel(const ArJoinParams P) {
  __shared__ float red[32];
  __shared__ int s_abort;
  __shared__ uint32_t s_epoch;
  __shared__ uint64_t s_target;
  const int tid = threadIdx.x;
  const uint64_t own = P.bufs[P.rank];
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(epoch_ptr(own, P)) + 1u;
    // the pushed calls' cumulative element count per source (plain calls leave it alone)
    s_target = *reinterpret_cast<volatile uint64_t*>(target_ptr(own, P)) +
               (P.pushed ? static_cast<uint64_t>(P.rows) * P.H : 0ull);
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int par = e & 1;
  const size_t slot_elems = static_cast<size_t>(P.rows_max) * P.H;

  if (P.pushed) {
    // the GEMM pushed every source's partial: wait until each source's element count reaches the target
    if (tid == 0) {
      for (int q = 0; q < P.world && !s_abort; ++q) {
        long long polls = 0;
        while (static_cast<int64_t>(ld_acquire_sys64(counter_ptr(own, P, q)) - s_target) < 0) {
          if (++polls > AR_MAX_POLLS) {
            s_abort = 1;
            flag_error(P.err, DEVERR_TIMEOUT);
            break;
          }
          __nanosleep(128);
        }
      }
    }
  } else {
    // 1. push this rank's rows into slot `rank` of every rank's buffer (own included)
    for (int row = blockIdx.x; row < P.rows; row += gridDim.x) push_row(P, row, par, slot_elems);
    __threadfence_system();
    __syncthreads();
    // 2. raise the rows' flags on every rank; 3. wait for every rank's flags of the rows on this rank (bounded)
    if (tid == 0) {
      for (int row = blockIdx.x; row < P.rows; row += gridDim.x)
        for (int q = 0; q < P.world; ++q) st_release_sys(flag_ptr(P.bufs[q], P, row, P.rank), e);
      for (int row = blockIdx.x; row < P.rows && !s_abort; row += gridDim.x) {
        for (int q = 0; q < P.world; ++q) {
          const uint32_t* f = flag_ptr(own, P, row, q);
          long long polls = 0;
          while (static_cast<int>(ld_acquire_sys(f) - e) < 0) {
            if (++polls > AR_MAX_POLLS) {
              s_abort = 1;
              flag_error(P.err, DEVERR_TIMEOUT);
              break;
            }
            __nanosleep(128);
          }
          if (s_abort) break;
        }
      }
    }
  }
  __syncthreads();
  __threadfence();
  const bool ok = !s_abort;

  // 4. per row: sum the world's slots in rank order, + residual; optional RMSNorm of the bf16 sum
  const bf16* slots0 = reinterpret_cast<const bf16*>(own) + static_cast<size_t>(par) * P.world * slot_elems;
  for (int row = blockIdx.x; row < P.rows; row += gridDim.x) {
    const float ss = reduce_row(P, row, slots0, slot_elems, ok);
    if (P.norm_w) {
      const float tot = block_sum(ss, red);  // its barriers also order this row's sum_out writes before the reads
      norm_row(P, row, rsqrtf(tot / static_cast<float>(P.H) + P.eps));
      __syncthreads();  // red is reused by the next row
    }
  }
  // 5. the last CTA to finish advances this rank's epoch for the next call
  __syncthreads();
  if (tid == 0) {
    uint32_t* done = epoch_ptr(own, P) + 1;
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0;
      if (P.pushed) *reinterpret_cast<volatile uint64_t*>(target_ptr(own, P)) = s_target;
      *reinterpret_cast<volatile uint32_t*>(epoch_ptr(own, P)) = e;
      __threadfence();
    }
  }
}

// ---- gated RMSNorm whose row statistic spans the ranks of a norm group (the Mamba-2 norm under tensor
// parallelism): each rank holds D columns of every row; the row's sum of squares of g = y * silu(z) is the sum
// of the ranks' partial sums. One kernel: partial sums pushed into every rank's buffer (slot [parity][rank][row],
// fp32), per-row flags as in the all-reduce, bounded waits, rank-order sum, then out = w * g * rsqrt(total /
// (world * D) + eps). Buffer: slots [2][world][rows_max] fp32, flags [rows_max][world] u32, epoch, done.
struct GnJoinParams {
  const uint64_t* bufs;
  int rank, world, rows_max, rows, D;
  const bf16* y; int64_t y_b;
  const bf16* z; int64_t z_b;
  const bf16* w;
  bf16* out; int64_t o_b;
  float eps;
  int* err;
};

__host__ __device__ inline size_t gn_flags_off(int world, int rows_max) { return 2ull * world * rows_max * 4; }
__host__ __device__ inline size_t gn_epoch_off(int world, int rows_max) {
  return gn_flags_off(world, rows_max) + static_cast<size_t>(rows_max) * world * 4;
}

__device__ __forceinline__ float gated(float y, float z) { return y * silu(z); }

__global__ void __launch_bounds__(AR_THREADS) gnorm_join_kernel(const GnJoinParams P) {
  __shared__ float red[32];
  __shared__ int s_abort;
  __shared__ uint32_t s_epoch;
  const int tid = threadIdx.x;
  const uint64_t own = P.bufs[P.rank];
  uint32_t* own_epoch = reinterpret_cast<uint32_t*>(own + gn_epoch_off(P.world, P.rows_max));
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(own_epoch) + 1u;
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int par = e & 1;
  const int nvec = P.D / 8;
  // 1. each row's partial sum of squares, pushed to every rank (thread 0) with the row's flag
  for (int row = blockIdx.x; row < P.rows; row += gridDim.x) {
    float ss = 0.f;
    for (int v = tid; v < nvec; v += AR_THREADS) {
      const uint4 yu = reinterpret_cast<const uint4*>(P.y + row * P.y_b)[v];
      const uint4 zu = reinterpret_cast<const uint4*>(P.z + row * P.z_b)[v];
      const uint32_t yw[4] = {yu.x, yu.y, yu.z, yu.w}, zw[4] = {zu.x, zu.y, zu.z, zu.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = unpack_bf16x2(yw[i]), b = unpack_bf16x2(zw[i]);
        const float g0 = gated(a.x, b.x), g1 = gated(a.y, b.y);
        ss = fmaf(g0, g0, fmaf(g1, g1, ss));
      }
    }
    const float tot = block_sum(ss, red);
    if (tid == 0) {
      for (int q = 0; q < P.world; ++q) {
        float* slot = reinterpret_cast<float*>(P.bufs[q]) + (static_cast<size_t>(par) * P.world + P.rank) * P.rows_max + row;
        *slot = tot;
      }
      __threadfence_system();
      for (int q = 0; q < P.world; ++q)
        st_release_sys(reinterpret_cast<uint32_t*>(P.bufs[q] + gn_flags_off(P.world, P.rows_max)) + row * P.world + P.rank, e);
    }
    __syncthreads();  // red is reused by the next row
  }
  // 2. wait for every rank's partial of this CTA's rows (bounded)
  if (tid == 0) {
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(own + gn_flags_off(P.world, P.rows_max));
    for (int row = blockIdx.x; row < P.rows && !s_abort; row += gridDim.x) {
      for (int q = 0; q < P.world; ++q) {
        long long polls = 0;
        while (static_cast<int>(ld_acquire_sys(flags + row * P.world + q) - e) < 0) {
          if (++polls > AR_MAX_POLLS) {
            s_abort = 1;
            flag_error(P.err, DEVERR_TIMEOUT);
            break;
          }
          __nanosleep(128);
        }
        if (s_abort) break;
      }
    }
  }
  __syncthreads();
  __threadfence();
  // 3. total in rank order, apply
  const float* slots = reinterpret_cast<const float*>(own) + static_cast<size_t>(par) * P.world * P.rows_max;
  for (int row = blockIdx.x; row < P.rows; row += gridDim.x) {
    float total = 0.f;
    if (!s_abort)
      for (int q = 0; q < P.world; ++q) total += __ldcg(slots + q * P.rows_max + row);
    const float r = rsqrtf(total / (static_cast<float>(P.world) * P.D) + P.eps);
    for (int v = tid; v < nvec; v += AR_THREADS) {
      const uint4 yu = reinterpret_cast<const uint4*>(P.y + row * P.y_b)[v];
      const uint4 zu = reinterpret_cast<const uint4*>(P.z + row * P.z_b)[v];
      const uint4 wu = reinterpret_cast<const uint4*>(P.w)[v];
      const uint32_t yw[4] = {yu.x, yu.y, yu.z, yu.w}, zw[4] = {zu.x, zu.y, zu.z, zu.w}, ww[4] = {wu.x, wu.y, wu.z, wu.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = unpack_bf16x2(yw[i]), b = unpack_bf16x2(zw[i]), c = unpack_bf16x2(ww[i]);
        o[i] = pack_bf16x2(c.x * gated(a.x, b.x) * r, c.y * gated(a.y, b.y) * r);
      }
      reinterpret_cast<uint4*>(P.out + row * P.o_b)[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  // 4. the last CTA advances the epoch
  __syncthreads();
  if (tid == 0) {
    uint32_t* done = own_epoch + 1;
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0;
      *reinterpret_cast<volatile uint32_t*>(own_epoch) = e;
      __threadfence();
    }
  }
}

// ---- CUDA IPC: export / import a device pointer as (allocation handle, offset)
using PFN_range = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
PFN_range g_range = nullptr;
std::mutex g_ipc_mu;
std::map<uintptr_t, uintptr_t> g_imported;  // pointer handed out -> base of the opened mapping

int get_range_fn() {
  if (g_range) return MMP_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || !fn) return mmp_set_error(MMP_ERR_CUDA, "cuMemGetAddressRange unavailable");
  g_range = reinterpret_cast<PFN_range>(fn);
  return MMP_OK;
}

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" size_t mmp_ar_buffer_bytes(int world, int rows_max, int H) { return ar_total_bytes(world, rows_max, H); }

extern "C" int mmp_ipc_export(const void* ptr, void* blob) {
  if (!ptr || !blob) return mmp_set_error(MMP_ERR_INVALID, "mmp_ipc_export: null pointer");
  int rc = get_range_fn();
  if (rc != MMP_OK) return rc;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ipc_export: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ipc_export: %s", cudaGetErrorString(e));
  const uint64_t off = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  memcpy(blob, &h, sizeof(h));
  memcpy(static_cast<char*>(blob) + sizeof(h), &off, sizeof(off));
  return MMP_OK;
}

extern "C" int mmp_ipc_import(const void* blob, void** ptr_out) {
  if (!blob || !ptr_out) return mmp_set_error(MMP_ERR_INVALID, "mmp_ipc_import: null pointer");
  cudaIpcMemHandle_t h;
  uint64_t off = 0;
  memcpy(&h, blob, sizeof(h));
  memcpy(&off, static_cast<const char*>(blob) + sizeof(h), sizeof(off));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ipc_import: %s", cudaGetErrorString(e));
  void* p = static_cast<char*>(base) + off;
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  g_imported[reinterpret_cast<uintptr_t>(p)] = reinterpret_cast<uintptr_t>(base);
  *ptr_out = p;
  return MMP_OK;
}

extern "C" int mmp_ipc_release(void* ptr) {
  uintptr_t base = 0;
  {
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    auto it = g_imported.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == g_imported.end()) return mmp_set_error(MMP_ERR_INVALID, "mmp_ipc_release: pointer was not imported");
    base = it->second;
    g_imported.erase(it);
  }
  cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ipc_release: %s", cudaGetErrorString(e));
  return MMP_OK;
}

extern "C" int mmp_ar_join(const uint64_t* bufs, int rank, int world, int rows_max, int pushed,
                           const void* part, int64_t p_b, const void* resid, int64_t r_b,
                           void* sum_out, int64_t s_b, const void* norm_w, float eps, void* norm_out, int64_t n_b,
                           int rows, int H, int* err, void* stream) {
  if (rows == 0) return MMP_OK;
  if (!bufs || (!pushed && !part) || !sum_out || (norm_w && !norm_out))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ar_join: null pointer");
  if (world < 1 || world > AR_MAX_WORLD || rank < 0 || rank >= world || rows < 0 || rows > rows_max || H <= 0 || H % 8)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ar_join: bad sizes rank=%d world=%d rows=%d rows_max=%d H=%d", rank,
                         world, rows, rows_max, H);
  auto rows_ok = [](const void* p, int64_t ld) { return !p || (aligned16(p) && ld % 8 == 0); };
  if (!rows_ok(part, p_b) || !rows_ok(resid, r_b) || !rows_ok(sum_out, s_b) || !rows_ok(norm_out, n_b) ||
      (norm_w && !aligned16(norm_w)))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ar_join: rows must be 16-byte aligned");
  ArJoinParams P{bufs, rank, world, rows, H, rows_max, pushed ? 1 : 0,
                 static_cast<const bf16*>(part), p_b, static_cast<const bf16*>(resid), r_b,
                 static_cast<bf16*>(sum_out), s_b, static_cast<const bf16*>(norm_w), eps,
                 static_cast<bf16*>(norm_out), n_b, err};
  // no programmatic dependent launch: the epoch this call reads is the one the previous call wrote at its end
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return mmp_set_error(MMP_ERR_INVALID, "mmp_ar_join: device %d", dev);
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows < sms[dev] ? rows : sms[dev]);
  cfg.blockDim = dim3(AR_THREADS);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaLaunchKernelEx(&cfg, ar_join_kernel, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ar_join: launch failed: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_ar_join");
}


extern "C" size_t mmp_gn_buffer_bytes(int world, int rows_max) {
  return (gn_epoch_off(world, rows_max) + 8 + 15) / 16 * 16;
}

extern "C" int mmp_gated_rmsnorm_p2p(const uint64_t* bufs, int rank, int world, int rows_max,
                                     const void* y, int64_t y_b, const void* z, int64_t z_b, const void* w,
                                     void* out, int64_t o_b, int rows, int D, float eps, int* err, void* stream) {
  if (rows == 0) return MMP_OK;
  if (!bufs || !y || !z || !w || !out) return mmp_set_error(MMP_ERR_INVALID, "mmp_gated_rmsnorm_p2p: null pointer");
  if (world < 1 || world > AR_MAX_WORLD || rank < 0 || rank >= world || rows < 0 || rows > rows_max || D <= 0 || D % 8)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gated_rmsnorm_p2p: bad sizes rank=%d world=%d rows=%d rows_max=%d D=%d",
                         rank, world, rows, rows_max, D);
  auto rows_ok = [](const void* p, int64_t ld) { return aligned16(p) && ld % 8 == 0; };
  if (!rows_ok(y, y_b) || !rows_ok(z, z_b) || !rows_ok(out, o_b) || !aligned16(w))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gated_rmsnorm_p2p: rows must be 16-byte aligned");
  GnJoinParams P{bufs, rank, world, rows_max, rows, D, static_cast<const bf16*>(y), y_b, static_cast<const bf16*>(z),
                 z_b, static_cast<const bf16*>(w), static_cast<bf16*>(out), o_b, eps, err};
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return mmp_set_error(MMP_ERR_INVALID, "mmp_gated_rmsnorm_p2p: device %d", dev);
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows < sms[dev] || sms[dev] <= 0 ? rows : sms[dev]);
  cfg.blockDim = dim3(AR_THREADS);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaLaunchKernelEx(&cfg, gnorm_join_kernel, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gated_rmsnorm_p2p: launch failed: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_gated_rmsnorm_p2p");
}
