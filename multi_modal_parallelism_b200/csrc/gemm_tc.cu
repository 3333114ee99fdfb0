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
#include "p2p_layout.cuh"
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace mmp {
namespace {

constexpr int TBM = 128, TBK = 64, TTHREADS = 128;

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
  PeerBufs push;  // decode output pushed into every rank's all-reduce buffer (push.bufs null: written to out)
};

template <int BN, int STAGES>
struct TcLayout {
  static constexpr int A_BYTES = TBM * TBK * 2;
  static constexpr int B_BYTES = BN * TBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int PIPE = STAGES * STAGE_BYTES;
  static constexpr int BARS = PIPE;                        // full[S], empty[S], done, recv: 8 bytes each
  static constexpr int TMEM_SLOT = BARS + 8 * (2 * STAGES + 2);
  static constexpr int ABORT = TMEM_SLOT + 4;
  static constexpr int USED = ABORT + 4;
  static constexpr int DYN = USED + 1024;                  // slack to align the ring to 1024 bytes
  // staged fp32 tile: plain tiles row-major [TBM][BN + 4]; swapped tiles column-major [BN][TBM + 4]
  static constexpr int SLD = BN + 4;
  static constexpr int TLD = TBM + 4;
  static_assert(TBM * SLD * 4 <= PIPE && BN * TLD * 4 <= PIPE, "the staged tile must fit in the ring");
  // split-K (swapped tiles) adds receive slots [ns][BN][rows_per], rows_per = round8(ceil(128 / ns)) <= 168 / ns
  // split-K over ns CTAs: each stages its tile as ns owner blocks [BN][rows_per] (OSTR floats apart, padded
  // so the two owners a warp writes fall in different banks) and receives ns blocks [ns][BN][rows_per]
  static __host__ __device__ constexpr int rows_per(int ns) { return ((TBM + ns - 1) / ns + 7) / 8 * 8; }
  static __host__ __device__ constexpr int ostr(int ns) { return BN * rows_per(ns) + 16; }
  static __host__ __device__ constexpr bool split_fits(int ns) {
    return (ns * ostr(ns) + ns * BN * rows_per(ns)) * 4 <= PIPE;
  }
};

// Instruction descriptor, kind::f16: bf16 A and B, fp32 accumulate, both K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t umma_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(TBM >> 4) << 24);
}

// Write 8 consecutive output elements (row r, columns c0..c0+7, the first n valid) = vals + addend.
__device__ __forceinline__ void store8(const TcParams& P, int r, int c0, const float* vals, int n) {
  bf16* dst = P.out + static_cast<int64_t>(r) * P.ldo + c0;
  const bf16* add = P.addend ? P.addend + static_cast<int64_t>(r) * P.ldd + c0 : nullptr;
  if (n == 8 && aligned16(dst) && (!add || aligned16(add))) {
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (add) {
      const uint4 u = *reinterpret_cast<const uint4*>(add);
      const float2 p0 = unpack_bf16x2(u.x), p1 = unpack_bf16x2(u.y), p2 = unpack_bf16x2(u.z), p3 = unpack_bf16x2(u.w);
      a[0] = p0.x; a[1] = p0.y; a[2] = p1.x; a[3] = p1.y; a[4] = p2.x; a[5] = p2.y; a[6] = p3.x; a[7] = p3.y;
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(vals[0] + a[0], vals[1] + a[1]), pack_bf16x2(vals[2] + a[2], vals[3] + a[3]),
                                                pack_bf16x2(vals[4] + a[4], vals[5] + a[5]), pack_bf16x2(vals[6] + a[6], vals[7] + a[7]));
    return;
  }
  for (int k = 0; k < n; ++k) dst[k] = f2bf(vals[k] + (add ? bf2f(add[k]) : 0.f));
}

// The same 8 output elements written into slot `rank` (parity par) of every rank's all-reduce buffer.
__device__ __forceinline__ void push8(const TcParams& P, int r, int c0, const float* vals, int n, int par) {
  const PeerBufs& B = P.push;
  if (n == 8 && (c0 & 7) == 0 && (B.H & 7) == 0) {
    const uint4 v = make_uint4(pack_bf16x2(vals[0], vals[1]), pack_bf16x2(vals[2], vals[3]), pack_bf16x2(vals[4], vals[5]),
                               pack_bf16x2(vals[6], vals[7]));
#pragma unroll 1
    for (int q = 0; q < B.world; ++q)
      *reinterpret_cast<uint4*>(ar_slot_elem(B.bufs[q], B, par, B.rank, r, c0)) = v;
    return;
  }
#pragma unroll 1
  for (int q = 0; q < B.world; ++q)
    for (int k = 0; k < n; ++k) *reinterpret_cast<bf16*>(ar_slot_elem(B.bufs[q], B, par, B.rank, r, c0 + k)) = f2bf(vals[k]);
}

// Sum `ns` staged fp32 blocks of tile rows [row0, row0 + nrows) (block q at src + q * src_stride; swapped
// tiles column-major [BN][ld], plain tiles row-major [nrows][ld]) and write them with the addend. Swapped:
// 8 consecutive tile rows are 8 consecutive output columns of one output row; plain: 8 consecutive columns of
// one tile row. Consecutive threads take consecutive chunks: 16-byte, coalesced, bank-conflict-free.
template <bool TRANS, int BN, bool PUSH = false>
__device__ __forceinline__ void finish_tile(const TcParams& P, const float* src, int ns, int src_stride, int ld,
                                            int row0, int nrows, int m0, int n0, int par = 0) {
  if (nrows <= 0) return;
  if constexpr (TRANS) {
    // source blocks are column-major [BN][ld]: tile rows g*8 .. g*8+7 of column c are two float4
    const int groups = (nrows + 7) / 8;
    for (int idx = threadIdx.x; idx < groups * BN; idx += TTHREADS) {
      const int g = idx % groups, c = idx / groups;
      const int orow = n0 + c, ocol = m0 + row0 + g * 8;
      if (orow >= P.b_rows) continue;
      const int n = min(8, min(nrows - g * 8, P.a_rows - ocol));
      if (n <= 0) continue;
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = 0.f;
      for (int q = 0; q < ns; ++q) {
        const float4* b = reinterpret_cast<const float4*>(src + q * src_stride + c * ld + g * 8);
        const float4 x = b[0], y = b[1];
        v[0] += x.x; v[1] += x.y; v[2] += x.z; v[3] += x.w; v[4] += y.x; v[5] += y.y; v[6] += y.z; v[7] += y.w;
      }
      if constexpr (PUSH) push8(P, orow, ocol, v, n, par);
      else store8(P, orow, ocol, v, n);
    }
  } else {
    constexpr int CH = BN / 8;
    for (int idx = threadIdx.x; idx < nrows * CH; idx += TTHREADS) {
      const int i = idx / CH, ch = idx % CH;
      const int orow = m0 + row0 + i, ocol = n0 + ch * 8;
      if (orow >= P.a_rows) continue;
      const int n = min(8, P.b_rows - ocol);
      if (n <= 0) continue;
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = 0.f;
      for (int q = 0; q < ns; ++q) {
        const float4* b = reinterpret_cast<const float4*>(src + q * src_stride + i * ld + ch * 8);
        const float4 x = b[0], y = b[1];
        v[0] += x.x; v[1] += x.y; v[2] += x.z; v[3] += x.w; v[4] += y.x; v[5] += y.y; v[6] += y.z; v[7] += y.w;
      }
      store8(P, orow, ocol, v, n);
    }
  }
}

template <int BN, int STAGES, bool TRANS, bool CLUSTER, bool PUSH = false>
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
  const uint32_t recv_bar = sbase + L::BARS + 8 * (2 * STAGES + 1);  // split-K partials received
  // swapped tiles scale each tile row (an output column) by the column scale: a weight-side constant, read
  // now so its latency hides under the main loop
  const int trow = warp * 32 + lane;
  const float cs_row = (TRANS && P.colscale && m0 + trow < P.a_rows) ? __ldg(P.colscale + m0 + trow) : 1.f;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::TMEM_SLOT);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(done_bar, 1);
    mbar_init(recv_bar, 1);
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

  // Output rows this CTA writes: split-K owners take rows_per tile rows each.
  int ns = 1, me = 0, rp = TBM;
  if constexpr (CLUSTER) {
    cg::cluster_group cluster = cg::this_cluster();
    ns = static_cast<int>(cluster.num_blocks());
    me = static_cast<int>(cluster.block_rank());
    rp = L::rows_per(ns);
  }
  const int own_row0 = me * rp, own_rows = max(0, min(rp, TBM - me * rp));

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
  } else if (warp >= 2) {
    // idle during the main loop: pull the addend this CTA adds in its epilogue into L2 (32-byte sectors)
    if (P.addend && own_rows > 0) {
      if constexpr (TRANS) {  // output rows n0 + c, columns m0 + own_row0 ..
        const int secs = (own_rows * 2 + 31) / 32;
        for (int i = tid - 64; i < BN * secs; i += 64) {
          const int c = i / secs, sc = i % secs;
          if (n0 + c < P.b_rows && m0 + own_row0 + sc * 16 < P.a_rows)
            prefetch_l2(P.addend + static_cast<int64_t>(n0 + c) * P.ldd + m0 + own_row0 + sc * 16);
        }
      } else {  // output rows m0 + i, columns n0 ..
        constexpr int SECS = BN * 2 / 32;
        for (int i = tid - 64; i < own_rows * SECS; i += 64) {
          const int rr = i / SECS, sc = i % SECS;
          if (m0 + own_row0 + rr < P.a_rows && n0 + sc * 16 < P.b_rows)
            prefetch_l2(P.addend + static_cast<int64_t>(m0 + own_row0 + rr) * P.ldd + n0 + sc * 16);
        }
      }
    }
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
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const bool have = ok && nkt > 0;

  // teardown of the ring: an aborted pipeline can leave copies in flight, so drain them. Otherwise the MMA
  // thread waited on every issued stage before the done barrier fired and nothing is left.
  if (tid == 0 && *abort_flag) {
    for (int i = max(0, issued - STAGES); i < issued; ++i) mbar_drain(full_bar(i % STAGES), (i / STAGES) & 1);
  }
  // pushed output: this call's parity, from the all-reduce epoch (written by the previous call's join kernel,
  // which completed before this kernel's dependency wait returned)
  __shared__ int s_par;
  if constexpr (PUSH) {
    if (tid == 0) {
      const PeerBufs& B = P.push;
      const uint32_t ep = *reinterpret_cast<volatile const uint32_t*>(B.bufs[B.rank] + ar_epoch_off(B.world, B.rows_max, B.H));
      s_par = static_cast<int>((ep + 1u) & 1u);
    }
  }
  __syncthreads();  // the ring is free: every MMA finished (done barrier), every copy landed (drain)

  // Stage the scaled fp32 tile in shared memory (tile row r = this thread's TMEM lane): alpha / alpha2 per K
  // segment and the column scale of the output column (a tile row when swapped, a tile column otherwise).
  float* stage = reinterpret_cast<float*>(smem);
  const int ostr = CLUSTER ? L::ostr(ns) : 0;
#pragma unroll 1
  for (int cb = 0; cb < BN; cb += 32) {
    // 32 accumulator columns per batch: both tcgen05.ld of an accumulator issued before one wait
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.f;
    if (have) {
      uint32_t t[32];
      if (has0) {
        tmem_ld16_nw(t_lane + cb, t);
        tmem_ld16_nw(t_lane + cb + 16, t + 16);
        tmem_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(t[j]) * P.alpha;
      }
      if (has1) {
        tmem_ld16_nw(t_lane + BN + cb, t);
        tmem_ld16_nw(t_lane + BN + cb + 16, t + 16);
        tmem_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaf(__uint_as_float(t[j]), P.alpha2, v[j]);
      }
    }
    if constexpr (TRANS && CLUSTER) {
      // owner-major blocks [owner][column][row within the owner's rows]
      float* dst = stage + (trow / rp) * ostr + trow % rp + cb * rp;
#pragma unroll
      for (int j = 0; j < 32; ++j) dst[j * rp] = v[j] * cs_row;
    } else if constexpr (TRANS) {
#pragma unroll
      for (int j = 0; j < 32; ++j) stage[(cb + j) * L::TLD + trow] = v[j] * cs_row;  // consecutive lanes: consecutive words
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int c = n0 + cb + j;
        if (P.colscale) v[j] *= c < P.b_rows ? P.colscale[c] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(stage + trow * L::SLD + cb + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
  }

  if constexpr (CLUSTER) {
    static_assert(TRANS, "split-K runs swapped (weight-streaming) tiles");
    // split-K reduce-scatter through distributed shared memory: owner o sums tile rows [o*rp, o*rp + rp).
    // Every CTA hands owner o its block with one bulk copy (copy engine) into the owner's receive slot for
    // it, completing on the owner's receive barrier; each owner then sums its ns slots.
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t blk_bytes = BN * rp * 4;
    const uint32_t recv_s = sbase + ns * ostr * 4;
    float* recv = stage + ns * ostr;  // [ns][BN][rp]
    if (tid == 0) mbar_expect_tx(recv_bar, ns * blk_bytes);
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // staged words -> the copy engine
    __syncthreads();
    cluster.sync();  // every CTA has staged its tile, stopped using its ring and armed its receive barrier
    if (tid == 0) {
      for (int o = 0; o < ns; ++o)
        bulk_s2cluster(mapa(recv_s + me * blk_bytes, o), sbase + o * ostr * 4, blk_bytes, mapa(recv_bar, o));
      asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
    }
    const bool got = mbar_wait(recv_bar, 0, abort_flag, P.err);
    if (got) finish_tile<TRANS, BN, PUSH>(P, recv, ns, BN * rp, rp, own_row0, own_rows, m0, n0, PUSH ? s_par : 0);
    if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");  // our blocks have left
  } else {
    __syncthreads();
    finish_tile<TRANS, BN, PUSH>(P, stage, 1, 0, TRANS ? L::TLD : L::SLD, 0, TBM, m0, n0, PUSH ? s_par : 0);
  }
  if constexpr (PUSH) {
    // every output element this CTA owns is in every rank's buffer: count them on every rank (release), so
    // the join kernel that follows knows when this rank's partial has fully arrived
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
      const PeerBufs& B = P.push;
      const int cols = max(0, min(own_rows, P.a_rows - (m0 + own_row0)));
      const int rows = max(0, min(BN, P.b_rows - n0));
      const uint64_t cnt = static_cast<uint64_t>(cols) * static_cast<uint64_t>(rows);
      if (cnt) {
        for (int q = 0; q < B.world; ++q) {
          uint64_t* c = reinterpret_cast<uint64_t*>(B.bufs[q] + ar_counters_off(B.world, B.rows_max, B.H)) + B.rank;
          asm volatile("red.release.sys.global.add.u64 [%0], %1;\n" ::"l"(c), "l"(cnt) : "memory");
        }
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

// ------------------------------------------------------------------------------------ persistent (prefill)
// Large M: one CTA per SM walks output tiles (tile t, t + gridDim.x, ...; N fastest, so the CTAs in flight
// share their A row panels and the whole weight stays in L2). Warp 0 lane 0 streams A/B boxes through the
// STAGES-deep ring across tile boundaries; warp 1 lane 0 issues the MMAs of tile i into TMEM accumulator
// buffer i % 2; warps 2-5 drain buffer (i-1) % 2 meanwhile (tcgen05.ld, scales, addend, 32-byte row stores)
// and hand it back through the acc_empty barrier. ACC = accumulators per tile (2 = two K segments).
constexpr int PTHREADS = 192;

template <int BN, int STAGES, int ACC>
struct PLayout {
  static constexpr int A_BYTES = TBM * TBK * 2;
  static constexpr int B_BYTES = BN * TBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int PIPE = STAGES * STAGE_BYTES;
  static constexpr int BARS = PIPE;  // full[S], empty[S], acc_full[2], acc_empty[2]
  static constexpr int TMEM_SLOT = BARS + 8 * (2 * STAGES + 4);
  static constexpr int ABORT = TMEM_SLOT + 4;
  static constexpr int USED = ABORT + 4;
  static constexpr int DYN = USED + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * ACC * BN;
  static_assert(TMEM_COLS <= 512, "two accumulator buffers must fit in TMEM");
};

template <int BN, int STAGES, int ACC>
__global__ void __launch_bounds__(PTHREADS, 1) gemm_tc_persistent(const __grid_constant__ CUtensorMap tmA,
                                                                 const __grid_constant__ CUtensorMap tmB,
                                                                 const TcParams P, int tiles_n, int ntiles) {
  using L = PLayout<BN, STAGES, ACC>;
  pdl_trigger();
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int k_tiles = (P.K + TBK - 1) / TBK;
  auto full_bar = [&](int s) { return sbase + L::BARS + 8 * s; };
  auto empty_bar = [&](int s) { return sbase + L::BARS + 8 * (STAGES + s); };
  auto accf_bar = [&](int b) { return sbase + L::BARS + 8 * (2 * STAGES + b); };
  auto acce_bar = [&](int b) { return sbase + L::BARS + 8 * (2 * STAGES + 2 + b); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::TMEM_SLOT);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), 4);  // one elected lane per epilogue warp
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(tmem_slot)), "r"(L::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int issued = 0;  // TMA stages issued by the producer (drained at teardown after an abort)
  if (warp == 0) {
    if (lane == 0) {
      // B (weights) never depends on the previous kernel: the first ring's worth of B boxes is requested
      // before waiting for it
      const int first = blockIdx.x;
      const int pre = first < ntiles ? min(k_tiles, STAGES) : 0;
      if (pre > 0) {
        const int n0 = (first % tiles_n) * BN;
        for (int i = 0; i < pre; ++i) {
          mbar_expect_tx(full_bar(i), L::STAGE_BYTES);
          tma_load_2d(sbase + i * L::STAGE_BYTES + L::A_BYTES, &tmB, full_bar(i), i * TBK, n0);
        }
      }
      pdl_wait();
      int kc = 0;
      for (int t = blockIdx.x; t < ntiles && !*abort_flag; t += gridDim.x) {
        const int m0 = (t / tiles_n) * TBM, n0 = (t % tiles_n) * BN;
        for (int kt = 0; kt < k_tiles; ++kt, ++kc) {
          const int s = kc % STAGES;
          const uint32_t a_s = sbase + s * L::STAGE_BYTES, b_s = a_s + L::A_BYTES;
          if (kc < pre) {  // B already requested
            tma_load_2d(a_s, &tmA, full_bar(s), kt * TBK, m0);
            ++issued;
            continue;
          }
          if (kc >= STAGES && !mbar_wait(empty_bar(s), ((kc / STAGES) - 1) & 1, abort_flag, P.err)) break;
          mbar_expect_tx(full_bar(s), L::STAGE_BYTES);
          tma_load_2d(a_s, &tmA, full_bar(s), kt * TBK, m0);
          tma_load_2d(b_s, &tmB, full_bar(s), kt * TBK, n0);
          ++issued;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      const uint32_t idesc = umma_idesc<BN>();
      int kc = 0, tc = 0;
      for (int t = blockIdx.x; t < ntiles && !*abort_flag; t += gridDim.x, ++tc) {
        const int buf = tc & 1;
        if (tc >= 2 && !mbar_wait(acce_bar(buf), ((tc >> 1) - 1) & 1, abort_flag, P.err)) break;
        tc_fence_after();
        bool started0 = false, started1 = false;
        bool ok = true;
        for (int kt = 0; kt < k_tiles; ++kt, ++kc) {
          const int s = kc % STAGES;
          if (!mbar_wait(full_bar(s), (kc / STAGES) & 1, abort_flag, P.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_s = sbase + s * L::STAGE_BYTES, b_s = a_s + L::A_BYTES;
          const bool seg1 = ACC == 2 && kt >= P.k_seg_tile;
          const uint32_t d = tmem + (buf * ACC + (seg1 ? 1 : 0)) * BN;
          const bool started = seg1 ? started1 : started0;
#pragma unroll
          for (int kk = 0; kk < TBK / 16; ++kk)
            umma_f16(d, umma_desc(a_s + kk * 32), umma_desc(b_s + kk * 32), idesc, started || kk != 0);
          if (seg1) started1 = true; else started0 = true;
          umma_commit(empty_bar(s));
        }
        if (!ok) break;
        umma_commit(accf_bar(buf));  // arrives once every MMA of this tile has completed
      }
    }
    __syncwarp();
  } else {
    // epilogue warps 2-5: warp w reads TMEM lanes 32 (w % 4) .. +31 = tile rows
    pdl_wait();
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const bool has0 = ACC == 1 || P.k_seg_tile > 0, has1 = ACC == 2 && P.k_seg_tile < k_tiles;
    int tc = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      const int buf = tc & 1;
      bool ok = mbar_wait(accf_bar(buf), (tc >> 1) & 1, abort_flag, P.err);
      ok = __all_sync(0xffffffffu, ok && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      const int m0 = (t / tiles_n) * TBM, n0 = (t % tiles_n) * BN;
      const int row = m0 + r;
      const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * ACC * BN;
#pragma unroll 1
      for (int cb = 0; cb < BN; cb += 16) {
        uint32_t a0[16], a1[16];
        if (has0) tmem_ld16_nw(t_lane + cb, a0);
        if (has1) tmem_ld16_nw(t_lane + BN + cb, a1);
        tmem_wait();
        if (row >= P.a_rows) continue;
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float x = has0 ? __uint_as_float(a0[j]) * P.alpha : 0.f;
          if (has1) x = fmaf(__uint_as_float(a1[j]), P.alpha2, x);
          v[j] = x;
        }
        const int c0 = n0 + cb;
        if (P.colscale) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] *= c0 + j < P.b_rows ? __ldg(P.colscale + c0 + j) : 0.f;
        }
        bf16* dst = P.out + static_cast<int64_t>(row) * P.ldo + c0;
        const bf16* add = P.addend ? P.addend + static_cast<int64_t>(row) * P.ldd + c0 : nullptr;
        if (c0 + 16 <= P.b_rows && aligned16(dst) && (!add || aligned16(add))) {
          if (add) {
            const uint4 u0 = reinterpret_cast<const uint4*>(add)[0], u1 = reinterpret_cast<const uint4*>(add)[1];
            const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float2 f = unpack_bf16x2(w[j]);
              v[2 * j] += f.x;
              v[2 * j + 1] += f.y;
            }
          }
          reinterpret_cast<uint4*>(dst)[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                        pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
          reinterpret_cast<uint4*>(dst)[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]),
                                                        pack_bf16x2(v[12], v[13]), pack_bf16x2(v[14], v[15]));
        } else {  // ragged right edge or unaligned rows
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < P.b_rows) dst[j] = f2bf(v[j] + (add ? bf2f(add[j]) : 0.f));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(acce_bar(buf)) : "memory");
    }
  }

  // teardown: after an abort the producer's copies may still be in flight
  if (tid == 0 && *abort_flag) {
    for (int i = max(0, issued - STAGES); i < issued; ++i) mbar_drain(full_bar(i % STAGES), (i / STAGES) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(L::TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------------------------- host side
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

template <int BN, int STAGES, bool TRANS, bool CLUSTER, bool PUSH = false>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const TcParams& P, dim3 grid, int split, cudaStream_t s) {
  using L = TcLayout<BN, STAGES>;
  auto kern = gemm_tc_kernel<BN, STAGES, TRANS, CLUSTER, PUSH>;
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

template <int BN, int STAGES, int ACC>
int launch_persistent(const CUtensorMap& ma, const CUtensorMap& mb, const TcParams& P, int tiles_n, int ntiles,
                      cudaStream_t s) {
  using L = PLayout<BN, STAGES, ACC>;
  auto kern = gemm_tc_persistent<BN, STAGES, ACC>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "gemm_tc: smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  const int grid = std::min(ntiles, g_tc_sms);
  cudaError_t e = mmp::launch_kind(1, kern, dim3(grid), dim3(PTHREADS), L::DYN, s, nullptr, 0, ma, mb, P, tiles_n, ntiles);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "gemm_tc: launch failed: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_gemm_bf16_tc");
}

int g_decode_split = 0;  // 0: the split-K count follows the rule below; > 0: that count (mmp_set_gemm_decode_split)
int g_decode_stages = 4;  // ring depth of the M <= 64 decode GEMMs: 4 (two CTAs per SM) or 8 (one per SM)

// Decode (M <= 256): swap-AB, A = weight rows (the 128-row M side of the MMA), B = the activation rows (N);
// K split over a cluster when the output tiles cannot fill the GPU. PUSH: output tiles go to every rank's
// all-reduce buffer (P.push) instead of P.out.
template <bool PUSH>
int decode_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, int M, int N, int K, TcParams& P, int k_tiles,
                cudaStream_t s) {
  int rc;
  CUtensorMap ma, mb;
  const int bn = M <= 64 ? 64 : 128;
  P.a_rows = N;
  P.b_rows = M;
  if ((rc = make_map(&ma, w, N, K, ldw, TBM)) || (rc = make_map(&mb, a, M, K, lda, bn))) return rc;
  const int tiles = (N + TBM - 1) / TBM;
  const int ntiles_b = (M + bn - 1) / bn;
  const bool deep = bn == 64 && g_decode_stages == 8;  // 8-stage ring: one CTA per SM, 192 KB of weights in flight
  const int slots = (bn == 64 && !deep ? 2 : 1) * g_tc_sms;  // CTAs that fit per SM at this tile shape
  int split = 1;
  if (tiles * ntiles_b < slots) split = std::min(8, std::max(1, std::min(slots / (tiles * ntiles_b), k_tiles / 2)));
  if (g_decode_split > 0) split = std::min(std::min(8, g_decode_split), std::max(1, k_tiles));  // a fixed count
  // the staged and received owner blocks must fit in the ring
  auto fits = [&](int ns) {
    return ns == 1 || (bn == 64 ? (deep ? TcLayout<64, 8>::split_fits(ns) : TcLayout<64, 4>::split_fits(ns))
                                : TcLayout<128, 5>::split_fits(ns));
  };
  int ktps = (k_tiles + split - 1) / split;
  split = (k_tiles + ktps - 1) / ktps;
  while (split > 1 && !fits(split)) {
    ktps = (k_tiles + split - 2) / (split - 1);
    split = (k_tiles + ktps - 1) / ktps;
  }
  P.k_tiles_per_split = ktps;
  dim3 grid(ntiles_b, tiles, split);
  const bool cl = split > 1;
  if (bn == 64 && deep)
    return cl ? launch_tc<64, 8, true, true, PUSH>(ma, mb, P, grid, split, s) : launch_tc<64, 8, true, false, PUSH>(ma, mb, P, grid, 1, s);
  if (bn == 64) return cl ? launch_tc<64, 4, true, true, PUSH>(ma, mb, P, grid, split, s) : launch_tc<64, 4, true, false, PUSH>(ma, mb, P, grid, 1, s);
  return cl ? launch_tc<128, 5, true, true, PUSH>(ma, mb, P, grid, split, s) : launch_tc<128, 5, true, false, PUSH>(ma, mb, P, grid, 1, s);
}

}  // namespace
}  // namespace mmp

using namespace mmp;

// The reference-named entry point (F.linear / @ and the layer's scalings, harness/kernels.py:147-154): the same
// tensor-core kernel without a device error word.
extern "C" int mmp_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int64_t ldo,
                             int M, int N, int K, float alpha, const float* colscale, const void* addend, int64_t ldd,
                             void* stream) {
  return mmp_gemm_bf16_tc(a, lda, w, ldw, out, ldo, M, N, K, alpha, colscale, addend, ldd, nullptr, stream);
}

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
  if (M <= 256) return decode_gemm<false>(a, lda, w, ldw, M, N, K, P, k_tiles, s);
  // large M (prefill): A = activations, B = weight rows; a persistent CTA per SM over 128 x 256 output tiles
  // (128 x 128 when two K segments need two accumulators per tile)
  P.a_rows = M;
  P.b_rows = N;
  const bool two = k_seg_tile < k_tiles;
  const int bn = two ? 128 : 256;
  if ((rc = make_map(&ma, a, M, K, lda, TBM)) || (rc = make_map(&mb, w, N, K, ldw, bn))) return rc;
  const int tiles_n = (N + bn - 1) / bn;
  const long long ntiles = static_cast<long long>(tiles_n) * ((M + TBM - 1) / TBM);
  if (ntiles > (1LL << 30)) return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16_tc: M=%d too large", M);
  if (two) return launch_persistent<128, 6, 2>(ma, mb, P, tiles_n, static_cast<int>(ntiles), s);
  return launch_persistent<256, 4, 1>(ma, mb, P, tiles_n, static_cast<int>(ntiles), s);
}

extern "C" int mmp_gemm_bf16_push(const void* a, int64_t lda, const void* w, int64_t ldw, int M, int N, int K,
                                  float alpha, int k_seg, float alpha2, const float* colscale, const uint64_t* bufs,
                                  int rank, int world, int rows_max, int* err, void* stream) {
  if (M == 0 || N == 0) return MMP_OK;
  if (!a || !w || !bufs) return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16_push: null pointer");
  if (M < 0 || M > 256 || M > rows_max || N < 0 || N % 8 || K <= 0 || K % 8 || lda % 8 || ldw % 8 || !aligned16(a) ||
      !aligned16(w) || lda < K || ldw < K || world < 1 || world > 8 || rank < 0 || rank >= world)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16_push: M=%d N=%d K=%d rows_max=%d rank=%d world=%d "
                         "(decode rows only; multiples of 8; 16-byte aligned)", M, N, K, rows_max, rank, world);
  if (k_seg < K && (k_seg <= 0 || k_seg % TBK))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16_push: k_seg %d must be a positive multiple of %d", k_seg, TBK);
  int rc = get_encoder();
  if (rc != MMP_OK) return rc;
  if (g_tc_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_tc_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_tc_sms <= 0) g_tc_sms = 148;
  }
  const int k_tiles = (K + TBK - 1) / TBK;
  const int k_seg_tile = k_seg < K ? k_seg / TBK : k_tiles;
  TcParams P{0, 0, K, k_tiles, nullptr, N, alpha, k_seg_tile, alpha2, colscale, nullptr, 0, err,
             PeerBufs{bufs, rank, world, rows_max, N}};
  return decode_gemm<true>(a, lda, w, ldw, M, N, K, P, k_tiles, static_cast<cudaStream_t>(stream));
}

extern "C" int mmp_set_gemm_decode_split(int split) {
  const int prev = mmp::g_decode_split;
  mmp::g_decode_split = split < 0 ? 0 : split;
  return prev;
}

extern "C" int mmp_set_gemm_decode_stages(int stages) {
  const int prev = mmp::g_decode_stages;
  mmp::g_decode_stages = stages == 8 ? 8 : 4;
  return prev;
}
