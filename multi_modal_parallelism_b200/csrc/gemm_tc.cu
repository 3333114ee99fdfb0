// bf16 GEMM on the 5th-generation tensor cores (tcgen05 / TMEM / TMA) for the layer's projections:
// out = alpha * colscale .* (x W^T) + addend (replaces F.linear / @ and the layer's scalings,
// harness/kernels.py:147-154 and harness/layer.py:35,80,105 of the reference).
//
// One CTA computes a 128 x BN fp32 tile D = A_tile . B_tile^T in TMEM, both operands K-major bf16:
//   * thread 0 streams 128x64 (A) and BNx64 (B) boxes with TMA (128-byte swizzle) into a STAGES-deep ring
//     guarded by full/empty mbarriers;
//   * thread 32 issues tcgen05.mma (M=128, N=BN, K=16, four per 64-wide k-tile) and releases each ring slot
//     with tcgen05.commit when the MMAs reading it are done;
//   * all 4 warps wait for the final commit, read their 32 TMEM lanes with tcgen05.ld and run the epilogue.
// Small M (decode, M = batch <= 256) runs "swap-AB": A = the weight (its rows are the 128-row MMA M side),
// B = the activations (N = batch), and the epilogue writes the transposed tile. When the output tiles cannot
// fill the GPU, K is split over up to 8 CTAs of a cluster whose fp32 partials are summed through distributed
// shared memory. Every mbarrier wait has a clock budget; a wait that runs out raises a CTA abort flag and the
// device error word, and teardown still drains in-flight copies and MMAs before TMEM is released.
#include <algorithm>
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>

#include "mmp_common.cuh"

namespace cg = cooperative_groups;

namespace mmp {
namespace {

constexpr int TBM = 128, TBK = 64, TTHREADS = 128;
constexpr long long WAIT_BUDGET_CYCLES = 4000000000LL;  // ~2 s at 2 GHz: far above any legitimate wait

struct TcParams {
  int a_rows, b_rows, K;
  int k_tiles_per_split;
  bf16* out; int64_t ldo;
  float alpha;
  int k_seg_tile;  // k-tiles from here on accumulate into a second TMEM accumulator scaled by alpha2
  float alpha2;
  const float* colscale;
  const bf16* addend; int64_t ldd;
  int* err;
};

template <int BN, int STAGES>
struct TcLayout {
  static constexpr int A_BYTES = TBM * TBK * 2;
  static constexpr int B_BYTES = BN * TBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int PIPE = STAGES * STAGE_BYTES;
  static constexpr int BARS = PIPE;                        // full[S], empty[S], done: 8 bytes each
  static constexpr int TMEM_SLOT = BARS + 8 * (2 * STAGES + 1);
  static constexpr int ABORT = TMEM_SLOT + 4;
  static constexpr int USED = ABORT + 4;
  static constexpr int DYN = USED + 1024;                  // slack to align the ring to 1024 bytes
  static constexpr int RLD4 = BN + 4;  // fp32 receive row (split-K): 16-byte aligned, conflict-free float4 columns
  static_assert((TBM + 8) * RLD4 * 4 <= PIPE, "split-K receive slots must fit in the ring");
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase completed; false when the CTA aborted or this wait ran out of budget.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > WAIT_BUDGET_CYCLES) {
      *abort_flag = 1;
      flag_error(err, DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];\n"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y) : "memory");
}

// UMMA shared-memory descriptor: K-major operand, 128-byte swizzle, 8-row core-matrix groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);          // start address
  d |= static_cast<uint64_t>(1) << 16;                          // leading byte offset (unused with swizzle)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;                  // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;                          // descriptor version (sm100)
  d |= static_cast<uint64_t>(2) << 61;                          // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: bf16 A and B, fp32 accumulate, both K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t umma_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(TBM >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

// 16 accumulator columns of this thread's TMEM lane, scaled: alpha * acc0 + alpha2 * acc1 (an accumulator
// this CTA never wrote contributes nothing). Warp-collective.
template <int BN>
__device__ __forceinline__ void load_scaled_bn(const TcParams& P, uint32_t taddr, bool has0, bool has1, float* v) {
  float a[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = 0.f;
  if (has0) {
    tmem_ld16(taddr, a);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = a[j] * P.alpha;
  }
  if (has1) {
    tmem_ld16(taddr + BN, a);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = fmaf(a[j], P.alpha2, v[j]);
  }
}
#define load_scaled(P, taddr, h0, h1, v) load_scaled_bn<BN>(P, taddr, h0, h1, v)

// out element (a_row i, b_row j): transposed tiles write out[j][i], plain tiles out[i][j]; colscale is
// indexed by the output column.
template <bool TRANS>
__device__ __forceinline__ void store_out(const TcParams& P, int i, int j, float scaled) {
  const int r = TRANS ? j : i, c = TRANS ? i : j;
  float v = scaled;
  if (P.colscale) v *= P.colscale[c];
  if (P.addend) v += bf2f(P.addend[static_cast<int64_t>(r) * P.ldd + c]);
  P.out[static_cast<int64_t>(r) * P.ldo + c] = f2bf(v);
}

template <int BN, int STAGES, bool TRANS, bool CLUSTER>
__global__ void __launch_bounds__(TTHREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                             const __grid_constant__ CUtensorMap tmB,
                                                             const TcParams P) {
  using L = TcLayout<BN, STAGES>;
  pdl_trigger();
  // Warp 0 (barrier set-up, TMEM allocation, TMA producer) waits for the previous kernel only once its lane 0
  // has started streaming the weight operand; warp-collective instructions stay convergent.
  if ((threadIdx.x >> 5) != 0) pdl_wait();
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.y * TBM;  // A rows
  const int n0 = blockIdx.x * BN;   // B rows
  const int k_tiles = (P.K + TBK - 1) / TBK;
  const int kt0 = blockIdx.z * P.k_tiles_per_split;
  const int nkt = max(0, min(k_tiles, kt0 + P.k_tiles_per_split) - kt0);
  // K segments: tiles [0, k_seg_tile) go to accumulator 0 (alpha), the rest to accumulator 1 (alpha2)
  const bool has0 = kt0 < min(kt0 + nkt, P.k_seg_tile), has1 = kt0 + nkt > max(kt0, P.k_seg_tile);
  const uint32_t tmem_cols = P.k_seg_tile < k_tiles ? 2 * BN : BN;
  auto full_bar = [&](int s) { return sbase + L::BARS + 8 * s; };
  auto empty_bar = [&](int s) { return sbase + L::BARS + 8 * (STAGES + s); };
  const uint32_t done_bar = sbase + L::BARS + 8 * (2 * STAGES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::TMEM_SLOT);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(tmem_slot)), "r"(tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Roles. The other lanes of the producer and MMA warps park at __syncwarp: a lane spinning in
  // mbarrier.try_wait can suspend its whole warp and starve the one lane that issues the copies or MMAs.
  int issued = 0;  // TMA stages issued by thread 0 (drained at teardown)
  if (warp == 0) {
    if (lane == 0) {
      // The weight operand (A when swapped for small M, else B) never depends on the previous kernel: its first
      // STAGES boxes are requested before waiting for that kernel, hiding their DRAM latency behind its tail.
      const int pre = min(nkt, STAGES);
      for (int i = 0; i < pre; ++i) {
        const uint32_t a_s = sbase + i * L::STAGE_BYTES, b_s = a_s + L::A_BYTES;
        mbar_expect_tx(full_bar(i), L::STAGE_BYTES);
        if (TRANS) tma_load_2d(a_s, &tmA, full_bar(i), (kt0 + i) * TBK, m0);
        else tma_load_2d(b_s, &tmB, full_bar(i), (kt0 + i) * TBK, n0);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const uint32_t a_s = sbase + i * L::STAGE_BYTES, b_s = a_s + L::A_BYTES;
        if (TRANS) tma_load_2d(b_s, &tmB, full_bar(i), (kt0 + i) * TBK, n0);
        else tma_load_2d(a_s, &tmA, full_bar(i), (kt0 + i) * TBK, m0);
      }
      issued = pre;
      for (int i = pre; i < nkt; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(empty_bar(s), ((i / STAGES) - 1) & 1, abort_flag, P.err)) break;
        const uint32_t a_s = sbase + s * L::STAGE_BYTES, b_s = a_s + L::A_BYTES;
        mbar_expect_tx(full_bar(s), L::STAGE_BYTES);
        const int kx = (kt0 + i) * TBK;
        tma_load_2d(a_s, &tmA, full_bar(s), kx, m0);
        tma_load_2d(b_s, &tmB, full_bar(s), kx, n0);
        ++issued;
      }
    }
    __syncwarp();
    if (lane != 0) pdl_wait();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc<BN>();
      bool started0 = false, started1 = false;
      for (int i = 0; i < nkt; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(full_bar(s), (i / STAGES) & 1, abort_flag, P.err)) break;
        tc_fence_after();
        const uint32_t a_s = sbase + s * L::STAGE_BYTES, b_s = a_s + L::A_BYTES;
        const int acc = kt0 + i >= P.k_seg_tile ? 1 : 0;
#pragma unroll
        for (int kk = 0; kk < TBK / 16; ++kk)
          umma_f16(tmem + acc * BN, umma_desc(a_s + kk * 32), umma_desc(b_s + kk * 32), idesc,
                   (acc ? started1 : started0) || kk != 0);
        if (acc) started1 = true; else started0 = true;
        umma_commit(empty_bar(s));
      }
      umma_commit(done_bar);  // arrives once every MMA issued above has completed
    }
    __syncwarp();
  }

  // epilogue: TMEM lane = A row (32 per warp), column = B row. tcgen05.ld is warp-collective: make the
  // go/no-go decision warp-uniform.
  bool ok = mbar_wait(done_bar, 0, abort_flag, P.err);
  ok = __all_sync(0xffffffffu, ok && !*abort_flag);
  tc_fence_after();
  const int arow = m0 + warp * 32 + lane;
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  if constexpr (!CLUSTER) {
    if (ok && nkt > 0) {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        load_scaled(P, t_lane + c0, has0, has1, v);
        if (arow < P.a_rows) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (n0 + c0 + j < P.b_rows) store_out<TRANS>(P, arow, n0 + c0 + j, v[j]);
        }
      }
    }
  }

  // teardown: drain this CTA's copies (an aborted pipeline can leave some in flight), then free TMEM
  if (tid == 0) {
    for (int i = 0; i < issued; ++i) {
      const int use = i / STAGES;
      if (i + STAGES >= issued) mbar_wait(full_bar(i % STAGES), use & 1, abort_flag, P.err);
    }
  }

  if constexpr (CLUSTER) {
    // split-K reduce-scatter through distributed shared memory: A rows are dealt to the cluster's CTAs in
    // contiguous blocks; every CTA pushes each of its rows (16-byte remote stores, no round trips) into the
    // owner's receive slot for that CTA, then each owner sums its rows' slots locally and runs the epilogue.
    cg::cluster_group cluster = cg::this_cluster();
    const int ns = static_cast<int>(cluster.num_blocks());
    const int me = static_cast<int>(cluster.block_rank());
    const int rows_per = (TBM + ns - 1) / ns;
    float* recv = reinterpret_cast<float*>(smem);  // [ns][rows_per][RLD4], overlays the drained ring
    const bool have = ok && nkt > 0;
    __syncthreads();
    cluster.sync();  // every CTA's ring is drained before anyone writes into it
    {
      const int row = warp * 32 + lane;
      const int owner = row / rows_per, rl = row % rows_per;
      float* dst = cluster.map_shared_rank(recv, owner) + (me * rows_per + rl) * L::RLD4;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        if (have) {
          load_scaled(P, t_lane + c0, has0, has1, v);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(dst + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
    }
    cluster.sync();  // all pushes have landed
    const int my_rows = min(rows_per, TBM - me * rows_per);
    for (int idx = tid; idx < my_rows * (BN / 4); idx += TTHREADS) {
      const int rl = idx % my_rows, c4 = idx / my_rows;  // consecutive threads: consecutive rows
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < ns; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(recv + (q * rows_per + rl) * L::RLD4 + c4 * 4);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const int i = m0 + me * rows_per + rl, j = n0 + c4 * 4;
      if (i < P.a_rows) {
        if (j < P.b_rows) store_out<TRANS>(P, i, j, acc.x);
        if (j + 1 < P.b_rows) store_out<TRANS>(P, i, j + 1, acc.y);
        if (j + 2 < P.b_rows) store_out<TRANS>(P, i, j + 2, acc.z);
        if (j + 3 < P.b_rows) store_out<TRANS>(P, i, j + 3, acc.w);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(tmem_cols));
  }
}

// ---------------------------------------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_encode_mu;

int get_encoder() {
  std::lock_guard<std::mutex> lock(g_encode_mu);
  if (g_encode) return MMP_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return mmp_set_error(MMP_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(e));
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return MMP_OK;
}

// 2-D K-major bf16 operand [rows, K] with row stride ld (elements), box of box_rows x 64.
int make_map(CUtensorMap* map, const void* base, int rows, int K, int64_t ld, int box_rows) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(TBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return mmp_set_error(MMP_ERR_INVALID, "tensor map encode failed (%d) rows=%d K=%d ld=%lld", (int)r, rows, K, (long long)ld);
  return MMP_OK;
}

int g_tc_sms = 0;

template <int BN, int STAGES, bool TRANS, bool CLUSTER>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const TcParams& P, dim3 grid, int split, cudaStream_t s) {
  using L = TcLayout<BN, STAGES>;
  auto kern = gemm_tc_kernel<BN, STAGES, TRANS, CLUSTER>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "gemm_tc: smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = split;
  cudaError_t e = mmp::launch_kind(1, kern, grid, dim3(TTHREADS), L::DYN, s, attr, CLUSTER ? 1 : 0, ma, mb, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "gemm_tc: launch failed: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_gemm_bf16_tc");
}

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" int mmp_gemm_bf16_tc(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int64_t ldo,
                                int M, int N, int K, float alpha, const float* colscale, const void* addend, int64_t ldd,
                                int* err, void* stream) {
  return mmp_gemm_bf16_seg(a, lda, w, ldw, out, ldo, M, N, K, alpha, K, alpha, colscale, addend, ldd, err, stream);
}

extern "C" int mmp_gemm_bf16_seg(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int64_t ldo,
                                 int M, int N, int K, float alpha, int k_seg, float alpha2, const float* colscale,
                                 const void* addend, int64_t ldd, int* err, void* stream) {
  if (M == 0 || N == 0) return MMP_OK;
  if (!a || !w || !out) return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16_tc: null pointer");
  if (M < 0 || N < 0 || K <= 0 || K % 8 || lda % 8 || ldw % 8 || !aligned16(a) || !aligned16(w) || lda < K ||
      ldw < K || ldo < N || (addend && ldd < N))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16_tc: M=%d N=%d K=%d lda=%lld ldw=%lld: K and strides must be "
                         "multiples of 8 with 16-byte aligned bases", M, N, K, (long long)lda, (long long)ldw);
  if (k_seg < K && (k_seg <= 0 || k_seg % TBK))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16_seg: k_seg %d must be a positive multiple of %d", k_seg, TBK);
  int rc = get_encoder();
  if (rc != MMP_OK) return rc;
  if (g_tc_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_tc_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_tc_sms <= 0) g_tc_sms = 148;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int k_tiles = (K + TBK - 1) / TBK;
  const int k_seg_tile = k_seg < K ? k_seg / TBK : k_tiles;
  TcParams P{0, 0, K, k_tiles, static_cast<bf16*>(out), ldo, alpha, k_seg_tile, alpha2, colscale,
             static_cast<const bf16*>(addend), ldd, err};
  CUtensorMap ma, mb;
  if (M <= 256) {
    // decode: swap-AB, A = weight rows (the 128-row M side of the MMA), B = the <= 256 activation rows
    const int bn = M <= 64 ? 64 : M <= 128 ? 128 : 256;
    P.a_rows = N;
    P.b_rows = M;
    if ((rc = make_map(&ma, w, N, K, ldw, TBM)) || (rc = make_map(&mb, a, M, K, lda, bn))) return rc;
    const int tiles = (N + TBM - 1) / TBM;
    const int slots = (bn == 64 ? 2 : 1) * g_tc_sms;  // CTAs that fit per SM at this tile shape
    int split = 1;
    if (tiles < slots) split = std::min(8, std::max(1, std::min(slots / tiles, k_tiles / 2)));
    const int ktps = (k_tiles + split - 1) / split;
    split = (k_tiles + ktps - 1) / ktps;
    P.k_tiles_per_split = ktps;
    dim3 grid(1, tiles, split);
    const bool cl = split > 1;
    switch (bn) {
      case 64: return cl ? launch_tc<64, 4, true, true>(ma, mb, P, grid, split, s) : launch_tc<64, 4, true, false>(ma, mb, P, grid, 1, s);
      case 128: return cl ? launch_tc<128, 4, true, true>(ma, mb, P, grid, split, s) : launch_tc<128, 4, true, false>(ma, mb, P, grid, 1, s);
      default: return cl ? launch_tc<256, 4, true, true>(ma, mb, P, grid, split, s) : launch_tc<256, 4, true, false>(ma, mb, P, grid, 1, s);
    }
  }
  // large M (prefill): A = activations, B = weight rows, 128 x 256 output tiles
  P.a_rows = M;
  P.b_rows = N;
  if ((rc = make_map(&ma, a, M, K, lda, TBM)) || (rc = make_map(&mb, w, N, K, ldw, 256))) return rc;
  dim3 grid((N + 255) / 256, (M + TBM - 1) / TBM, 1);
  if (grid.y > 65535) return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16_tc: M=%d too large", M);
  return launch_tc<256, 4, false, false>(ma, mb, P, grid, 1, s);
}
