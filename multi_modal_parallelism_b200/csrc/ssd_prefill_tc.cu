// Mamba-2 prefill chunked scan on the 5th-generation tensor cores (tcgen05 / TMEM / TMA), head dim 128 and
// d_state 128 or 256; the restated algorithm and its reference citations are in ssd_prefill.cu, which keeps
// the other shapes.
//
// One CTA (8 warps) owns one head of one sequence and walks its chunks of 64 tokens in order. The fp32 state
// S [p = 128, N] lives in TMEM for the whole walk (lane = p, column = n). Per chunk, with cum the running sum
// of dt' A inside the chunk:
//   * TMA brings C, B [64 x N] and x [64 x 128] (128-byte swizzle, K-major boxes); the next chunk's boxes are
//     prefetched into L2 meanwhile;
//   * G = C B^T (tcgen05.mma M=64, N=64, K=N) into TMEM; meanwhile the threads write the bf16 copy of S to
//     shared memory and exp(cum_last) S back to TMEM;
//   * the threads turn G into M[t][s] = G exp(cum_t - cum_s) dt_s (s <= t), plus D on the diagonal (so the
//     intra-chunk product carries the D x skip term), and scale B rows by w_s = exp(cum_last - cum_s) dt_s
//     in place;
//   * y^T = x^T M^T and ys^T = S C^T into two TMEM accumulators (M=128 over p, N=64 over t), combined as
//     y = y + exp(cum_t) ys in the epilogue; S += x^T (w B) (M=128, N=N); x and B are read as MN-major
//     operands straight from their TMA boxes, M, C and the bf16 S as K-major ones;
//   * once the MMAs are done the next chunk's loads go out, and the y tile is staged and written (16-byte
//     stores) under them.
// Every mbarrier wait is bounded (tc_common.cuh); a CTA that runs out of budget flags the error word, leaves
// its state line untouched, drains its copies and frees TMEM.
#include <algorithm>

#include "mmp_common.cuh"
#include "tc_common.cuh"

namespace mmp {
namespace {

constexpr int SQ = 64;     // tokens per chunk
constexpr int SP = 128;    // head dim handled by this kernel
constexpr int STHR = 256;  // 8 warps

struct SsdTcParams {
  const bf16* dt; int64_t dt_t, dt_h;
  const float* A; const float* D; const float* dt_bias;
  void* state; int64_t s_line, s_head, s_p;
  const int32_t* cu_seqlens; const int32_t* state_idx; const int32_t* has_init;
  bf16* out; int64_t o_t, o_h;
  int nh, ngroups, lines;
  int* err;
};

template <int N>
struct TcSsdSmem {
  static constexpr int KB = N / 64;                   // 64-wide k-blocks along n
  static constexpr int C_OFF = 0;                     // C chunk: KB blocks [64 t x 128 B]
  static constexpr int B_OFF = C_OFF + KB * 8192;     // B chunk: same
  static constexpr int X_OFF = B_OFF + KB * 8192;     // x chunk: 2 blocks [64 t x 128 B] (p 0-63, 64-127)
  static constexpr int M_OFF = X_OFF + 2 * 8192;      // M: [64 t x 128 B] (s)
  static constexpr int SB_OFF = M_OFF + 8192;         // bf16 S: KB blocks [128 p x 128 B]
  static constexpr int YLD = SP * 2 + 16;             // y tile row bytes (padded)
  static constexpr int Y_OFF = SB_OFF + KB * 16384;   // y tile [64 t][128 p] bf16
  static constexpr int CUM_OFF = Y_OFF + SQ * YLD;    // cum[64], dt[64], w[64], exp(cum)[64] fp32
  static constexpr int BAR_OFF = CUM_OFF + 4 * SQ * 4 + 16;
  static constexpr int USED = BAR_OFF + 8 * 4 + 16;
  static constexpr int DYN = USED + 1024;
  static constexpr uint32_t LOAD_BYTES = 2 * KB * 8192 + 2 * 8192;
};

// TMEM columns
constexpr uint32_t T_S = 0, T_Y = 256, T_G = 320, T_YS = 384;

// byte offset of 16-byte chunk c of row r in a 128-byte-swizzled block of 128-byte rows
__device__ __forceinline__ uint32_t sw(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// UMMA shared-memory descriptor of an MN-major operand stored as TMA boxes [K rows][64 MN elements] (128-byte
// swizzle): 8-row K groups 1024 bytes apart (stride byte offset), 64-element MN blocks `mn_block` bytes apart
// (leading byte offset)
__device__ __forceinline__ uint64_t umma_desc_mn(uint32_t saddr, uint32_t mn_block) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>((mn_block >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
constexpr uint32_t IDESC_A_MN = 1u << 15, IDESC_B_MN = 1u << 16;

// bf16 copy of 64 state columns (this thread's row p) into the K-major operand blocks of the state term
template <int N>
__device__ __forceinline__ void store_sb(uint8_t* smem, int p, int c0n, const uint32_t* r) {
  uint8_t* rowp = smem + TcSsdSmem<N>::SB_OFF + (c0n >> 6) * 16384;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(rowp + sw(p, c)) = make_uint4(
        pack_bf16x2(__uint_as_float(r[8 * c + 0]), __uint_as_float(r[8 * c + 1])),
        pack_bf16x2(__uint_as_float(r[8 * c + 2]), __uint_as_float(r[8 * c + 3])),
        pack_bf16x2(__uint_as_float(r[8 * c + 4]), __uint_as_float(r[8 * c + 5])),
        pack_bf16x2(__uint_as_float(r[8 * c + 6]), __uint_as_float(r[8 * c + 7])));
}

template <typename ST, int N>
__global__ void __launch_bounds__(STHR, 1) ssd_prefill_tc_kernel(const __grid_constant__ CUtensorMap mapX,
                                                                const __grid_constant__ CUtensorMap mapB,
                                                                const __grid_constant__ CUtensorMap mapC,
                                                                const SsdTcParams P) {
  using L = TcSsdSmem<N>;
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
  pdl_trigger();
  pdl_wait();
  const uint32_t sb = smem_addr(smem);
  const int h = blockIdx.x, seq = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, half = warp >> 2;
  const int t_begin = P.cu_seqlens[seq], t_end = P.cu_seqlens[seq + 1];
  const int line = P.state_idx[seq];
  if (line < 0 || line >= P.lines) {
    if (tid == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const int grp = h / (P.nh / P.ngroups);
  const float A = P.A[h], Dh = P.D ? P.D[h] : 0.f, dtb = P.dt_bias ? P.dt_bias[h] : 0.f;
  float* sCum = reinterpret_cast<float*>(smem + L::CUM_OFF);
  float* sDt = sCum + SQ;
  float* sW = sDt + SQ;
  float* sE = sW + SQ;    // exp(cum_t)
  float* sDec = sE + SQ;  // exp(cum_last)
  const uint32_t bar_load = sb + L::BAR_OFF, bar_g = bar_load + 8, bar_y = bar_load + 16, bar_s = bar_load + 24;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::BAR_OFF + 32);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + 36);
  ST* gstate = reinterpret_cast<ST*>(P.state) + line * P.s_line + h * P.s_head;

  if (tid == 0) {
    mbar_init(bar_load, 1);
    mbar_init(bar_g, 1);
    mbar_init(bar_y, 1);
    mbar_init(bar_s, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&mapX)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&mapB)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&mapC)) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(smem_addr(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // this thread's TMEM lane (= state / output row p) and its half of the columns
  const int p = q * 32 + lane;
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16);

  // ---- initial state into TMEM (or zeros) and its bf16 copy for the first chunk's state term
  {
    const bool init = P.has_init && P.has_init[seq];
#pragma unroll 1
    for (int c0n = half * (N / 2); c0n < (half + 1) * (N / 2); c0n += 64) {
      uint32_t r[64];
#pragma unroll
      for (int j = 0; j < 64; ++j)
        r[j] = __float_as_uint(init ? static_cast<float>(gstate[p * P.s_p + c0n + j]) : 0.f);
#pragma unroll
      for (int k = 0; k < 4; ++k) tmem_st16(t_lane + T_S + c0n + 16 * k, r + 16 * k);
      store_sb<N>(smem, p, c0n, r);
    }
    tmem_wait_st();
  }

  auto issue_loads = [&](int c0) {
    mbar_expect_tx(bar_load, L::LOAD_BYTES);
#pragma unroll
    for (int kb = 0; kb < L::KB; ++kb) {
      tma_load_3d(sb + L::C_OFF + kb * 8192, &mapC, bar_load, kb * 64, grp, c0);
      tma_load_3d(sb + L::B_OFF + kb * 8192, &mapB, bar_load, kb * 64, grp, c0);
    }
    tma_load_3d(sb + L::X_OFF, &mapX, bar_load, 0, h, c0);
    tma_load_3d(sb + L::X_OFF + 8192, &mapX, bar_load, 64, h, c0);
    if (c0 + SQ < t_end) {  // the chunk after into L2
#pragma unroll
      for (int kb = 0; kb < L::KB; ++kb) {
        tma_prefetch_3d(&mapC, kb * 64, grp, c0 + SQ);
        tma_prefetch_3d(&mapB, kb * 64, grp, c0 + SQ);
      }
      tma_prefetch_3d(&mapX, 0, h, c0 + SQ);
      tma_prefetch_3d(&mapX, 64, h, c0 + SQ);
    }
  };
  if (tid == 0 && t_begin < t_end) issue_loads(t_begin);

  bool ok = true;  // warp-uniform: this warp's last wait succeeded (loop exits follow the CTA's abort flag)
  int it = 0;
  for (int c0 = t_begin; c0 < t_end; c0 += SQ, ++it) {
    const int qn = min(SQ, t_end - c0);
    const uint32_t par = it & 1;
    if (warp == 1) {
      // dt' = softplus(dt + bias), inclusive running sum of dt' A, state-update weights, chunk decay
      float d[2], cs[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = lane * 2 + j;
        d[j] = r < qn ? softplus(bf2f(P.dt[static_cast<int64_t>(c0 + r) * P.dt_t + h * P.dt_h]) + dtb) : 0.f;
      }
      cs[0] = d[0] * A;
      cs[1] = cs[0] + d[1] * A;
      float run = cs[1];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, run, o);
        if (lane >= o) run += v;
      }
      const float excl = run - cs[1];
      const float cum_last = __shfl_sync(0xffffffffu, run, 31);  // tokens past qn add nothing
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = lane * 2 + j;
        const float cum = excl + cs[j];
        sDt[r] = d[j];
        sCum[r] = cum;
        sW[r] = r < qn ? __expf(cum_last - cum) * d[j] : 0.f;
        sE[r] = __expf(cum);
      }
      if (lane == 0) *sDec = __expf(cum_last);
    }
    mbar_wait(bar_load, par, abort_flag, P.err);
    __syncthreads();  // scan results visible; a thread whose wait ran out raised the flag before arriving
    if (*abort_flag) break;

    // ---- G = C B^T (M = 64 tokens t, N = 64 tokens s, K = n)
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t idg = umma_idesc_mn(64, 64);
#pragma unroll
      for (int kb = 0; kb < L::KB; ++kb)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem + T_G, umma_desc(sb + L::C_OFF + kb * 8192 + kk * 32),
                   umma_desc(sb + L::B_OFF + kb * 8192 + kk * 32), idg, (kb | kk) != 0);
      umma_commit(bar_g);
    }

    // ---- meanwhile: the state decays in TMEM, S = exp(cum_last) S (its bf16 copy, made at the end of the
    // previous chunk, keeps the incoming state for the state term)
    {
      const float dec = *sDec;
#pragma unroll 1
      for (int c0n = half * (N / 2); c0n < (half + 1) * (N / 2); c0n += 64) {
        uint32_t r[64];
#pragma unroll
        for (int k = 0; k < 4; ++k) tmem_ld16_nw(t_lane + T_S + c0n + 16 * k, r + 16 * k);
        tmem_wait();
#pragma unroll
        for (int j = 0; j < 64; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * dec);
#pragma unroll
        for (int k = 0; k < 4; ++k) tmem_st16(t_lane + T_S + c0n + 16 * k, r + 16 * k);
      }
      tmem_wait_st();
    }

    // ---- G -> M (masked, decayed, dt-weighted, D on the diagonal); B rows *= w_s
    ok = mbar_wait(bar_g, par, abort_flag, P.err);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      // M=64 accumulator: row t = 16 q + l sits in lane 32 q + l (l < 16) of quadrant q; warps 0-3 take
      // columns 0-31, warps 4-7 columns 32-63
      uint32_t g[32];
      tmem_ld16_nw(t_lane + T_G + half * 32, g);
      tmem_ld16_nw(t_lane + T_G + half * 32 + 16, g + 16);
      tmem_wait();
      if (lane < 16) {
        const int t = q * 16 + lane;
        const float ct = sCum[t];
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint32_t w4[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int s0 = half * 32 + c8 * 8 + 2 * j;
            const int jj = c8 * 8 + 2 * j;
            float a = (s0 <= t && s0 < qn) ? __uint_as_float(g[jj]) * __expf(ct - sCum[s0]) * sDt[s0] : 0.f;
            float b = (s0 + 1 <= t && s0 + 1 < qn) ? __uint_as_float(g[jj + 1]) * __expf(ct - sCum[s0 + 1]) * sDt[s0 + 1] : 0.f;
            if (s0 == t) a += Dh;
            if (s0 + 1 == t) b += Dh;
            w4[j] = pack_bf16x2(a, b);
          }
          *reinterpret_cast<uint4*>(smem + L::M_OFF + sw(t, half * 4 + c8)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // M -> tensor core reads
    tc_fence_before();
    __syncthreads();  // M built; the G MMAs are done with B (every thread passed bar_g)
    if (*abort_flag) break;

    // ---- y^T = x^T M^T ; ys^T = S C^T (B is not an operand: it is weighted meanwhile)
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t idy_x = umma_idesc_mn(128, 64) | IDESC_A_MN;
      constexpr uint32_t idy = umma_idesc_mn(128, 64);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)  // K = s, 16 rows of the x boxes per step
        umma_f16(tmem + T_Y, umma_desc_mn(sb + L::X_OFF + kk * 2048, 8192), umma_desc(sb + L::M_OFF + kk * 32),
                 idy_x, kk != 0);
#pragma unroll
      for (int kb = 0; kb < L::KB; ++kb)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem + T_YS, umma_desc(sb + L::SB_OFF + kb * 16384 + kk * 32),
                   umma_desc(sb + L::C_OFF + kb * 8192 + kk * 32), idy, (kb | kk) != 0);
      umma_commit(bar_y);
    }
    if (ok) {
      // row t = tid / 4 of B, a quarter of its 16-byte chunks each
      const int t = tid >> 2, part = tid & 3;
      const float wb = sW[t];
#pragma unroll
      for (int i = 0; i < L::KB * 2; ++i) {
        const int cidx = part * (L::KB * 2) + i;  // chunk along n: block cidx / 8, chunk cidx % 8
        uint4* pb = reinterpret_cast<uint4*>(smem + L::B_OFF + (cidx >> 3) * 8192 + sw(t, cidx & 7));
        const uint4 v = *pb;
        const float2 a0 = unpack_bf16x2(v.x), a1 = unpack_bf16x2(v.y), a2 = unpack_bf16x2(v.z), a3 = unpack_bf16x2(v.w);
        *pb = make_uint4(pack_bf16x2(a0.x * wb, a0.y * wb), pack_bf16x2(a1.x * wb, a1.y * wb),
                         pack_bf16x2(a2.x * wb, a2.y * wb), pack_bf16x2(a3.x * wb, a3.y * wb));
      }
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic smem writes -> tensor core reads
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) break;

    // ---- S += x^T (w B)
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t ids = umma_idesc_mn(128, N) | IDESC_A_MN | IDESC_B_MN;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_f16(tmem + T_S, umma_desc_mn(sb + L::X_OFF + kk * 2048, 8192),
                 umma_desc_mn(sb + L::B_OFF + kk * 2048, 8192), ids, 1);
      umma_commit(bar_s);
    }

    // ---- y^T out of TMEM; once the state update is done too, the next chunk's loads go out and the y tile is
    // staged and stored under them
    ok = mbar_wait(bar_y, par, abort_flag, P.err);
    ok = __all_sync(0xffffffffu, ok);
    float yv[32];
    if (ok) {
      tc_fence_after();
      uint32_t yi[32], ys[32];
      tmem_ld16_nw(t_lane + T_Y + half * 32, yi);
      tmem_ld16_nw(t_lane + T_Y + half * 32 + 16, yi + 16);
      tmem_ld16_nw(t_lane + T_YS + half * 32, ys);
      tmem_ld16_nw(t_lane + T_YS + half * 32 + 16, ys + 16);
      tmem_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) yv[j] = fmaf(sE[half * 32 + j], __uint_as_float(ys[j]), __uint_as_float(yi[j]));
    }
    mbar_wait(bar_s, par, abort_flag, P.err);
    tc_fence_after();
    __syncthreads();  // every MMA of this chunk is done: C, B, x, M and the bf16 S are free
    if (*abort_flag) break;
    if (tid == 0 && c0 + SQ < t_end) issue_loads(c0 + SQ);
    // bf16 copy of the outgoing state (the next chunk's state term) while the loads are in flight
#pragma unroll 1
    for (int c0n = half * (N / 2); c0n < (half + 1) * (N / 2); c0n += 64) {
      uint32_t r[64];
#pragma unroll
      for (int k = 0; k < 4; ++k) tmem_ld16_nw(t_lane + T_S + c0n + 16 * k, r + 16 * k);
      tmem_wait();
      store_sb<N>(smem, p, c0n, r);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j)
      *reinterpret_cast<bf16*>(smem + L::Y_OFF + (half * 32 + j) * L::YLD + p * 2) = f2bf(yv[j]);
    __syncthreads();
    for (int i = tid; i < SQ * (SP / 8); i += STHR) {
      const int t = i / (SP / 8), c = i % (SP / 8);
      if (t < qn)
        st16(P.out + static_cast<int64_t>(c0 + t) * P.o_t + h * P.o_h + c * 8,
             *reinterpret_cast<const uint4*>(smem + L::Y_OFF + t * L::YLD + c * 16));
    }
    // the y tile is rewritten after the next chunk's loads and MMAs, each behind a barrier
  }

  // ---- final state -> the sequence's line (skipped after an abort: the line keeps its old value)
  const bool aborted = *abort_flag != 0;
  if (!aborted) {
#pragma unroll 1
    for (int c0n = half * (N / 2); c0n < (half + 1) * (N / 2); c0n += 16) {
      uint32_t r[16];
      tmem_ld16_nw(t_lane + T_S + c0n, r);
      tmem_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) gstate[p * P.s_p + c0n + j] = static_cast<ST>(__uint_as_float(r[j]));
    }
  } else if (tid == 0) {
    // copies of the chunk that was loading may still be in flight
    mbar_drain(bar_load, it & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem));
  }
}

// 3-D tensor map over [T rows][mid][inner] bf16 (row stride s_t, middle stride s_mid, elements), box 64 x 1 x 64
int make_map3(CUtensorMap* map, const void* base, int inner, int mid, int rows, int64_t s_mid, int64_t s_t) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(mid), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s_mid) * 2, static_cast<cuuint64_t>(s_t) * 2};
  cuuint32_t box[3] = {64, 1, 64};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: tensor map encode failed (%d)", (int)r);
  return MMP_OK;
}

template <typename ST, int N>
int launch_ssd_tc(const CUtensorMap& mx, const CUtensorMap& mb, const CUtensorMap& mc, const SsdTcParams& P, int nseq,
                  cudaStream_t s) {
  using L = TcSsdSmem<N>;
  auto kern = ssd_prefill_tc_kernel<ST, N>;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssd_prefill: smem attribute: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  cudaError_t e = mmp::launch(kern, dim3(P.nh, nseq), dim3(STHR), L::DYN, s, nullptr, 0, mx, mb, mc, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssd_prefill: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_ssd_prefill");
}

}  // namespace

// The tensor-core path for head dim 128, d_state 128 / 256 with TMA-compatible strides; MMP_UNSUPPORTED
// otherwise (the caller then runs the mma.sync kernel).
int ssd_prefill_tc(const void* x, int64_t x_t, int64_t x_h, const void* dt, int64_t dt_t, int64_t dt_h, const float* A,
                   const float* D, const float* dt_bias, const void* B, int64_t B_t, int64_t B_g, const void* C,
                   int64_t C_t, int64_t C_g, void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                   const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init, void* out,
                   int64_t o_t, int64_t o_h, int nseq, int ntok, int nh, int p, int N, int ngroups, int lines, int* err,
                   cudaStream_t stream) {
  if (p != SP || (N != 128 && N != 256) || ntok <= 0 || nh > 65535 || nseq > 65535) return MMP_ERR_UNSUPPORTED;
  if (x_h % 8 || x_t % 8 || B_g % 8 || B_t % 8 || C_g % 8 || C_t % 8 || !aligned16(x) || !aligned16(B) ||
      !aligned16(C) || o_t % 8 || o_h % 8 || !aligned16(out) || s_p < N)
    return MMP_ERR_UNSUPPORTED;
  int rc = get_encoder();
  if (rc != MMP_OK) return rc;
  CUtensorMap mx, mb, mc;
  if ((rc = make_map3(&mx, x, SP, nh, ntok, x_h, x_t)) || (rc = make_map3(&mb, B, N, ngroups, ntok, B_g, B_t)) ||
      (rc = make_map3(&mc, C, N, ngroups, ntok, C_g, C_t)))
    return rc;
  SsdTcParams P{static_cast<const bf16*>(dt), dt_t, dt_h, A, D, dt_bias, state, s_line, s_head, s_p,
                cu_seqlens, state_idx, has_init, static_cast<bf16*>(out), o_t, o_h, nh, ngroups, lines, err};
  const bool f32 = state_dtype == MMP_F32;
  if (N == 256) return f32 ? launch_ssd_tc<float, 256>(mx, mb, mc, P, nseq, stream) : launch_ssd_tc<bf16, 256>(mx, mb, mc, P, nseq, stream);
  return f32 ? launch_ssd_tc<float, 128>(mx, mb, mc, P, nseq, stream) : launch_ssd_tc<bf16, 128>(mx, mb, mc, P, nseq, stream);
}

}  // namespace mmp
