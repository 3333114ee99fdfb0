// Mamba-2 prefill chunked scan on the 5th-generation tensor cores (tcgen05 / TMEM / TMA), head dim 128 and
// d_state 128 or 256; the restated algorithm and its reference citations are in ssd_prefill.cu, which keeps
// the other shapes.
//
// One CTA owns one head of one sequence and walks its chunks of 64 tokens in order. The fp32 state S [p = 128, N]
// lives in TMEM for the whole walk (lane = p, column = n). Per chunk, with cum the running sum of dt' A inside the
// chunk, the work is split over warp roles that run concurrently:
//   * warp 8: one thread streams C, B [64 x N] and x [64 x 128] of each chunk through a two-stage ring of
//     128-byte-swizzled TMA boxes, a chunk ahead of the math; then the whole warp runs the chunk's scan of dt
//     (softplus, running sum, update weights, decays) into a four-deep ring of small shared-memory buffers;
//   * warp 9 (one thread) issues the MMAs: G = C B^T (M = 64 t, N = 64 s, K = N); Y = x^T M^T and
//     YS = S_bf C^T (M = 128 p, N = 64 t; the second reads the bf16 copy of the incoming state straight from TMEM
//     as its A operand, and shares its TMEM columns with G); S += (w x)^T B (M = 128 p, N = N);
//   * warps 0-3 (one state row p per thread): the weighted copy w x of the chunk's x rows (w_s = exp(cum_last -
//     cum_s) dt_s; double-buffered, made while the previous update still runs), then, once that update is done,
//     the state pass: the bf16 copy of S into TMEM and exp(cum_last) S back into the fp32 columns;
//   * warps 4-7 turn G into M[t][s] = G exp(cum_t - cum_s) dt_s (s <= t, D on the diagonal, so the product also
//     carries the D x skip term), all 128 lanes on 32 elements each; read Y and YS out of TMEM as soon as they
//     are done, build the next chunk's M, and then y = Y + exp(cum_t) YS is staged as bf16 and stored with
//     16-byte writes.
// The critical path per chunk is the update MMA, the state pass and the next Y and update MMAs; loads, the scan,
// the weighted x, G, the M build and the y stores run under them. Every mbarrier wait is bounded (tc_common.cuh); a CTA
// that runs out of budget flags the error word, leaves its state line untouched, drains its copies and MMAs and
// frees TMEM.
#include <algorithm>

#include "mmp_common.cuh"
#include "tc_common.cuh"

namespace mmp {
namespace {

constexpr int SQ = 64;     // tokens per chunk
constexpr int SP = 128;    // head dim handled by this kernel
constexpr int STHR = 320;  // warps 0-3 state pass, 4-7 scan / M / y, 8 copies, 9 MMAs

struct SsdTcParams {
  const bf16* dt; int64_t dt_t, dt_h;
  const float* A; const float* D; const float* dt_bias;
  void* state; int64_t s_line, s_head, s_p;
  const int32_t* cu_seqlens; const int32_t* state_idx; const int32_t* has_init;
  bf16* out; int64_t o_t, o_h;
  int nh, ngroups, lines;
  int* err;
};

// HP = heads per CTA: 1 for head dim 128; 2 for head dim 64, two heads of one B/C group stacked in the 128 TMEM lanes
// (lane = 64 h + p). With two heads the chunk's x is stored as the block-diagonal MN-major operand of Y = x^T M^T over
// K = (head, s): [x of head 0 | zeros | zeros | x of head 1], 8 KB each, so one K = 128 MMA chain applies each head's
// own M (the zero blocks are written once; the loads never touch them).
template <int N, int HP>
struct TcSsdSmem {
  static constexpr int KB = N / 64;                   // 64-wide k-blocks along n
  static constexpr int X_BYTES = 2 * 8192 * HP;
  static constexpr int STAGE = 2 * KB * 8192 + X_BYTES;  // one chunk's C, B and x boxes
  static constexpr int C_OFF = 0;                     // stage 0 C chunk: KB blocks [64 t x 128 B]
  static constexpr int B_OFF = C_OFF + KB * 8192;     // stage 0 B chunk: same
  static constexpr int X_OFF = B_OFF + KB * 8192;     // stage 0 x chunk: 2 blocks [64 t x 128 B] (p 0-63, 64-127)
  static constexpr int X_HEAD = 8192 + 16384 * (HP - 1);  // offset of the second block / head's x
  static constexpr int M_OFF = 2 * STAGE;             // M: per head [64 t x 128 B] (s)
  static constexpr int YLD = SP * 2 + 16;             // y tile row bytes (padded)
  static constexpr int Y_OFF = M_OFF + HP * 8192;     // y tile [64 t][128 p] bf16
  static constexpr int XW_OFF = Y_OFF + SQ * YLD;     // w-weighted x, per chunk parity: 2 blocks [64 t x 128 B]
  static constexpr int CUM_OFF = XW_OFF + 2 * 16384;  // per chunk (ring of 4), per head: cum log2e, dt, w, exp(cum) [64] + decay
  static constexpr int CUM_HEAD = 4 * SQ * 4 + 16;
  static constexpr int CUM_BYTES = HP * CUM_HEAD;
  static constexpr int BAR_OFF = CUM_OFF + 4 * CUM_BYTES;
  static constexpr int NBAR = 16;
  static constexpr int USED = BAR_OFF + 8 * NBAR + 16;
  static constexpr int DYN = USED + 1024;
  static constexpr uint32_t LOAD_BYTES = 2 * KB * 8192 + 2 * 8192;  // the zero blocks are not loaded
};
static_assert(TcSsdSmem<256, 1>::DYN <= 232448 && TcSsdSmem<128, 2>::DYN <= 232448, "shared memory per CTA");

// TMEM columns: fp32 state [N], bf16 state copy [N / 2] (two values per column), Y [64], and G / YS [64] (G is read
// out before YS is written into the same columns, and YS before the next G)
template <int N>
struct TcSsdTmem {
  static constexpr uint32_t S = 0, SBF = N, Y = N + N / 2, G = N + N / 2 + 64, YS = G;
};
static_assert(TcSsdTmem<256>::G + 64 <= 512, "TMEM columns");

// mbarriers
// (B_SCAN + i: the scan results in ring slot i are written; phase = chunk / 4, so no waiter can fall two phases
// behind: a slot is rewritten only after every reader of its previous chunk is done)
constexpr int B_FULL = 0, B_EMPTY = 2, B_G = 4, B_MB = 5, B_YFREE = 7, B_Y = 8, B_S = 9, B_SCAN = 10, B_DONE = 14;

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

// MMA with the A operand in TMEM (K-major, two bf16 per 32-bit column, lane = row)
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
      ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mbar_arrive1(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ float ex2f(float x) {  // 2^x on the MUFU unit (ex2.approx.ftz)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// AND of `v` over the `nthreads` threads of named barrier `id` (a barrier for them too): a decision every warp of
// a group takes alike, so that none leaves a loop while the others wait at the group's next barrier
__device__ __forceinline__ bool bar_and(int id, int nthreads, bool v) {
  int r;
  asm volatile("{\n.reg .pred p, q;\nsetp.ne.s32 p, %1, 0;\nbar.red.and.pred q, %2, %3, p;\nselp.s32 %0, 1, 0, q;\n}\n"
               : "=r"(r) : "r"(v ? 1 : 0), "r"(id), "r"(nthreads) : "memory");
  return r != 0;
}
// 64 consecutive TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t* r) {
#pragma unroll
  for (int k = 0; k < 4; ++k) tmem_ld16_nw(taddr + 16 * k, r + 16 * k);
}

template <typename ST, int N, int HP>
__global__ void __launch_bounds__(STHR, 1) ssd_prefill_tc_kernel(const __grid_constant__ CUtensorMap mapX,
                                                                const __grid_constant__ CUtensorMap mapB,
                                                                const __grid_constant__ CUtensorMap mapC,
                                                                const SsdTcParams P) {
  using L = TcSsdSmem<N, HP>;
  using TM = TcSsdTmem<N>;
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
  pdl_trigger();
  pdl_wait();
  const uint32_t sb = smem_addr(smem);
  const int h = blockIdx.x * HP, seq = blockIdx.y;  // the CTA's (first) head
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t_begin = P.cu_seqlens[seq], t_end = P.cu_seqlens[seq + 1];
  const int line = P.state_idx[seq];
  if (line < 0 || line >= P.lines) {
    if (tid == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const int nchunks = (t_end - t_begin + SQ - 1) / SQ;
  const int grp = h / (P.nh / P.ngroups);
  float A_[HP], D_[HP], dtb_[HP];
#pragma unroll
  for (int hh = 0; hh < HP; ++hh) {
    A_[hh] = P.A[h + hh];
    D_[hh] = P.D ? P.D[h + hh] : 0.f;
    dtb_[hh] = P.dt_bias ? P.dt_bias[h + hh] : 0.f;
  }
  auto bar = [&](int i) { return sb + L::BAR_OFF + 8 * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::BAR_OFF + 8 * L::NBAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + 8 * L::NBAR + 4);
  // this thread's state row when it is a state-pass thread (tid < 128: lane = head hh * 64 + row)
  ST* gstate = reinterpret_cast<ST*>(P.state) + line * P.s_line + (h + (HP == 2 ? (tid & 127) / 64 : 0)) * P.s_head;
  // per-chunk scan results, a ring of four (chunk c's buffer is rewritten by chunk c + 4, whose loads wait for
  // chunk c + 2's MMAs, which come after every reader of chunk c's buffer): cum log2(e), dt', w, exp(cum), decay
  auto cum_buf = [&](int c, int hh) {
    return reinterpret_cast<float*>(smem + L::CUM_OFF + (c & 3) * L::CUM_BYTES + hh * L::CUM_HEAD);
  };
  if constexpr (HP == 2) {  // the zero blocks of the block-diagonal x operand, both stages (before the first MMA)
    for (int i = tid; i < 2 * 2 * 8192 / 16; i += STHR) {
      const int stg = i / 1024, blk = (i / 512) & 1, off = (i & 511) * 16;
      *reinterpret_cast<uint4*>(smem + stg * L::STAGE + L::X_OFF + 8192 + blk * 8192 + off) = make_uint4(0u, 0u, 0u, 0u);
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  }

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(B_FULL + s), 1);
      mbar_init(bar(B_EMPTY + s), 1);
    }
    mbar_init(bar(B_G), 1);
    mbar_init(bar(B_MB), 256);
    mbar_init(bar(B_YFREE), 128);
    mbar_init(bar(B_Y), 1);
    mbar_init(bar(B_S), 1);
    for (int i = 0; i < 4; ++i) mbar_init(bar(B_SCAN + i), 32);
    mbar_init(bar(B_DONE), 1);
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

  if (warp == 8) {
    // ------------------------------------------------------------------ copies (one thread), then the scan (warp)
    int issued = 0;
    for (int c = 0; c < nchunks; ++c) {
      const int s = c & 1;
      const int c0 = t_begin + c * SQ;
      int go = 1;
      if (lane == 0) {
        if (c >= 2 && !mbar_wait(bar(B_EMPTY + s), ((c >> 1) - 1) & 1, abort_flag, P.err)) go = 0;
        if (*abort_flag) go = 0;
        if (go) {
          const uint32_t st = sb + s * L::STAGE;
          mbar_expect_tx(bar(B_FULL + s), L::LOAD_BYTES);
#pragma unroll
          for (int kb = 0; kb < L::KB; ++kb) {
            tma_load_3d(st + L::C_OFF + kb * 8192, &mapC, bar(B_FULL + s), kb * 64, grp, c0);
            tma_load_3d(st + L::B_OFF + kb * 8192, &mapB, bar(B_FULL + s), kb * 64, grp, c0);
          }
          // x: p 0-63 and 64-127 of the head, or the two heads (64 each) into the block-diagonal operand
          tma_load_3d(st + L::X_OFF, &mapX, bar(B_FULL + s), 0, h, c0);
          tma_load_3d(st + L::X_OFF + L::X_HEAD, &mapX, bar(B_FULL + s), HP == 1 ? 64 : 0, h + HP - 1, c0);
          if (c + 2 < nchunks) {  // the chunk after next into L2
#pragma unroll
            for (int kb = 0; kb < L::KB; ++kb) {
              tma_prefetch_3d(&mapC, kb * 64, grp, c0 + 2 * SQ);
              tma_prefetch_3d(&mapB, kb * 64, grp, c0 + 2 * SQ);
            }
            tma_prefetch_3d(&mapX, 0, h, c0 + 2 * SQ);
            tma_prefetch_3d(&mapX, HP == 1 ? 64 : 0, h + HP - 1, c0 + 2 * SQ);
          }
          issued = c + 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      // the scan: dt' = softplus(dt + bias), inclusive running sum of dt' A (kept times log2(e) for ex2), update
      // weights w, exp(cum) and the chunk decay exp(cum_last)
      const int qn = min(SQ, t_end - c0);
#pragma unroll
      for (int hh = 0; hh < HP; ++hh) {
        const float A = A_[hh], dtb = dtb_[hh];
        float* sCum = cum_buf(c, hh);
        float* sDt = sCum + SQ;
        float* sW = sDt + SQ;
        float* sE = sW + SQ;
        float d[2], cs[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int r = lane * 2 + j;
          d[j] = r < qn ? softplus(bf2f(P.dt[static_cast<int64_t>(c0 + r) * P.dt_t + (h + hh) * P.dt_h]) + dtb) : 0.f;
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
          sCum[r] = cum * 1.4426950408889634f;
          sW[r] = r < qn ? __expf(cum_last - cum) * d[j] : 0.f;
          sE[r] = __expf(cum);
        }
        if (lane == 0) sCum[4 * SQ] = __expf(cum_last);
      }
      mbar_arrive1(bar(B_SCAN + (c & 3)));
    }
    // copies in flight may still land after an abort: wait (bounded) for the last chunk of each stage
    if (lane == 0)
      for (int c = max(0, issued - 2); c < issued; ++c) mbar_drain(bar(B_FULL + (c & 1)), (c >> 1) & 1);
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMAs (one thread)
    if (lane == 0) {
      constexpr uint32_t idg = umma_idesc_mn(64, 64);
      constexpr uint32_t idy_x = umma_idesc_mn(128, 64) | IDESC_A_MN;
      constexpr uint32_t idy_s = umma_idesc_mn(128, 64);
      constexpr uint32_t ids = umma_idesc_mn(128, N) | IDESC_A_MN | IDESC_B_MN;
      auto issue_g = [&](int c) {  // G = C B^T (M = 64 tokens t, N = 64 tokens s, K = n)
        const uint32_t st = sb + (c & 1) * L::STAGE;
#pragma unroll
        for (int kb = 0; kb < L::KB; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + TM::G, umma_desc(st + L::C_OFF + kb * 8192 + kk * 32),
                     umma_desc(st + L::B_OFF + kb * 8192 + kk * 32), idg, (kb | kk) != 0);
        umma_commit(bar(B_G));
      };
      bool ok = nchunks > 0 && mbar_wait(bar(B_FULL), 0, abort_flag, P.err);
      if (ok) {
        tc_fence_after();
        issue_g(0);
      }
      for (int c = 0; ok && c < nchunks; ++c) {
        const uint32_t par = c & 1;
        const uint32_t st = sb + (c & 1) * L::STAGE;
        // M built, the state pass done and B weighted; Y and YS of the previous chunk read out
        if (!(ok = mbar_wait(bar(B_MB), par, abort_flag, P.err))) break;
        if (c > 0 && !(ok = mbar_wait(bar(B_YFREE), par ^ 1, abort_flag, P.err))) break;
        tc_fence_after();
        // Y = x^T M^T (K = s; with two heads K = (head, s) over the block-diagonal x and the heads' M side by side);
        // YS = S_bf C^T (K = n), into G's columns (G is read out)
#pragma unroll
        for (int kb = 0; kb < HP; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + TM::Y, umma_desc_mn(st + L::X_OFF + kb * 8192 + kk * 2048, HP == 1 ? 8192 : 16384),
                     umma_desc(sb + L::M_OFF + kb * 8192 + kk * 32), idy_x, (kb | kk) != 0);
#pragma unroll
        for (int kb = 0; kb < L::KB; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ts(tmem + TM::YS, tmem + TM::SBF + kb * 32 + kk * 8,
                        umma_desc(st + L::C_OFF + kb * 8192 + kk * 32), idy_s, (kb | kk) != 0);
        umma_commit(bar(B_Y));
        // S += (w x)^T B (K = t)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem + TM::S, umma_desc_mn(sb + L::XW_OFF + (c & 1) * 16384 + kk * 2048, 8192),
                   umma_desc_mn(st + L::B_OFF + kk * 2048, 8192), ids, 1);
        umma_commit(bar(B_S));
        umma_commit(bar(B_EMPTY + (c & 1)));  // every MMA reading this stage has been issued
        if (c + 1 < nchunks) {  // the next chunk's G, once YS is read out of its columns
          if (!(ok = mbar_wait(bar(B_YFREE), par, abort_flag, P.err))) break;
          if (!(ok = mbar_wait(bar(B_FULL + ((c + 1) & 1)), ((c + 1) >> 1) & 1, abort_flag, P.err))) break;
          tc_fence_after();
          issue_g(c + 1);
        }
      }
      umma_commit(bar(B_DONE));  // arrives once every MMA issued above has completed
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------------ warps 0-3: the state in TMEM, B weights
    const int p = HP == 1 ? tid : (tid & 63);  // state row of this thread's head (TMEM lane = tid)
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const bool init = P.has_init && P.has_init[seq];
#pragma unroll 1
    for (int c0n = 0; c0n < N; c0n += 16) {
      uint32_t r[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(init ? static_cast<float>(gstate[p * P.s_p + c0n + j]) : 0.f);
      tmem_st16(t_lane + TM::S + c0n, r);
    }
    tmem_wait_st();
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      const uint32_t par = c & 1;
      // this chunk's scan results and x tile: the weighted copy w x (row t = p / 2, one 64-wide block each)
      ok = mbar_wait(bar(B_SCAN + (c & 3)), (c >> 2) & 1, abort_flag, P.err) &&
           mbar_wait(bar(B_FULL + (c & 1)), (c >> 1) & 1, abort_flag, P.err);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      const float* sCum = cum_buf(c, HP == 1 ? 0 : tid / 64);
      {
        // one 64-wide block each: p 0-63 / 64-127 of the head, or one of the two heads (its own weights)
        const int t = tid >> 1, blk = tid & 1;
        const float wt = cum_buf(c, HP == 1 ? 0 : blk)[2 * SQ + t];
        const uint8_t* xs = smem + (c & 1) * L::STAGE + L::X_OFF + blk * L::X_HEAD;
        uint8_t* xd = smem + L::XW_OFF + (c & 1) * 16384 + blk * 8192;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint4 v = *reinterpret_cast<const uint4*>(xs + sw(t, k));
          const float2 a0 = unpack_bf16x2(v.x), a1 = unpack_bf16x2(v.y), a2 = unpack_bf16x2(v.z),
                       a3 = unpack_bf16x2(v.w);
          *reinterpret_cast<uint4*>(xd + sw(t, k)) =
              make_uint4(pack_bf16x2(a0.x * wt, a0.y * wt), pack_bf16x2(a1.x * wt, a1.y * wt),
                         pack_bf16x2(a2.x * wt, a2.y * wt), pack_bf16x2(a3.x * wt, a3.y * wt));
        }
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic smem writes -> tensor core reads
      if (c > 0) ok = mbar_wait(bar(B_S), par ^ 1, abort_flag, P.err);  // the previous update done
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      const float dec = sCum[4 * SQ];
      // bf16 copy of the incoming state (YS's A operand) and the decayed state (the update accumulates on it)
#pragma unroll 1
      for (int c0n = 0; c0n < N; c0n += 64) {
        uint32_t r[64], b[32];
        tmem_ld64(t_lane + TM::S + c0n, r);
        tmem_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) b[j] = pack_bf16x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
#pragma unroll
        for (int j = 0; j < 64; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * dec);
#pragma unroll
        for (int k = 0; k < 4; ++k) tmem_st16(t_lane + TM::S + c0n + 16 * k, r + 16 * k);
        tmem_st16(t_lane + TM::SBF + c0n / 2, b);
        tmem_st16(t_lane + TM::SBF + c0n / 2 + 16, b + 16);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive1(bar(B_MB));
    }
    // final state -> the sequence's line (skipped after an abort: the line keeps its old value)
    if (ok && nchunks > 0) ok = mbar_wait(bar(B_S), (nchunks - 1) & 1, abort_flag, P.err);
    ok = __all_sync(0xffffffffu, ok) && !*abort_flag;
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c0n = 0; c0n < N; c0n += 16) {
        uint32_t r[16];
        tmem_ld16_nw(t_lane + TM::S + c0n, r);
        tmem_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) gstate[p * P.s_p + c0n + j] = static_cast<ST>(__uint_as_float(r[j]));
      }
    }
  } else {
    // ------------------------------------------------------------------ warps 4-7: M, then y
    const int tl = tid - 128;  // 0..127
    const int q = warp & 3;    // TMEM lane quadrant
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(q * 32) << 16);
    // G(c) -> M(c). The M=64 accumulator puts row t = 16 q + l in lane 32 q + l (l < 16) of quadrant q: lanes l and
    // l + 16 share row t, columns 0-31 and 32-63 (the upper half passed over by a shuffle). False when a wait
    // ran out (the same on every warp of the group).
    auto build_m = [&](int c) -> bool {
      const bool ok = mbar_wait(bar(B_SCAN + (c & 3)), (c >> 2) & 1, abort_flag, P.err) &&
                      mbar_wait(bar(B_G), c & 1, abort_flag, P.err);
      if (!bar_and(2, 128, ok)) return false;
      tc_fence_after();
      uint32_t g[64];
      tmem_ld64(t_lane + TM::G, g);
      tmem_wait();
      tc_fence_before();  // G's columns are rewritten (YS) after the arrive below
      const int l16 = lane & 15, cb = lane >= 16 ? 32 : 0;
      const int t = q * 16 + l16;
      float gv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float hi = __uint_as_float(__shfl_sync(0xffffffffu, g[32 + j], l16));
        gv[j] = lane >= 16 ? hi : __uint_as_float(g[j]);
      }
#pragma unroll
      for (int hh = 0; hh < HP; ++hh) {  // the head's own decays on the group's shared C B^T
        const float* sCum = cum_buf(c, hh);
        const float* sDt = sCum + SQ;
        const float Dh = D_[hh];
        const float ct = sCum[t];
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          const float4 cs0 = *reinterpret_cast<const float4*>(sCum + cb + c8 * 8);
          const float4 cs1 = *reinterpret_cast<const float4*>(sCum + cb + c8 * 8 + 4);
          const float4 dt0 = *reinterpret_cast<const float4*>(sDt + cb + c8 * 8);
          const float4 dt1 = *reinterpret_cast<const float4*>(sDt + cb + c8 * 8 + 4);
          const float csv[8] = {cs0.x, cs0.y, cs0.z, cs0.w, cs1.x, cs1.y, cs1.z, cs1.w};
          const float dtv[8] = {dt0.x, dt0.y, dt0.z, dt0.w, dt1.x, dt1.y, dt1.z, dt1.w};
          float m[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int sidx = cb + c8 * 8 + e;
            // s <= t only: for s > t the exponent is positive and may overflow. dt' is 0 past the sequence
            m[e] = sidx <= t ? gv[c8 * 8 + e] * ex2f(ct - csv[e]) * dtv[e] : 0.f;
            if (sidx == t) m[e] += Dh;
          }
          *reinterpret_cast<uint4*>(smem + L::M_OFF + hh * 8192 + sw(t, (cb >> 3) + c8)) =
              make_uint4(pack_bf16x2(m[0], m[1]), pack_bf16x2(m[2], m[3]), pack_bf16x2(m[4], m[5]),
                         pack_bf16x2(m[6], m[7]));
        }
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic smem writes -> tensor core reads
      tc_fence_before();
      mbar_arrive1(bar(B_MB));
      return true;
    };
    if (nchunks > 0 && build_m(0)) {
      for (int c = 0; c < nchunks; ++c) {
        const int c0 = t_begin + c * SQ;
        const int qn = min(SQ, t_end - c0);
        // y = Y + exp(cum_t) YS out of TMEM (lane p, column t), kept as bf16 pairs while the next M is built
        if (!bar_and(2, 128, mbar_wait(bar(B_Y), c & 1, abort_flag, P.err))) break;
        tc_fence_after();
        uint32_t yp[32];
        {
          uint32_t yv[64], ys[64];
          tmem_ld64(t_lane + TM::Y, yv);
          tmem_ld64(t_lane + TM::YS, ys);
          tmem_wait();
          tc_fence_before();
          mbar_arrive1(bar(B_YFREE));  // Y and YS may be overwritten
          const float* sE = cum_buf(c, HP == 1 ? 0 : q / 2) + 3 * SQ;  // lanes 64 h .. 64 h + 63: head h
#pragma unroll
          for (int j4 = 0; j4 < 16; ++j4) {
            const float4 e = *reinterpret_cast<const float4*>(sE + 4 * j4);
            yp[2 * j4] = pack_bf16x2(fmaf(e.x, __uint_as_float(ys[4 * j4]), __uint_as_float(yv[4 * j4])),
                                     fmaf(e.y, __uint_as_float(ys[4 * j4 + 1]), __uint_as_float(yv[4 * j4 + 1])));
            yp[2 * j4 + 1] =
                pack_bf16x2(fmaf(e.z, __uint_as_float(ys[4 * j4 + 2]), __uint_as_float(yv[4 * j4 + 2])),
                            fmaf(e.w, __uint_as_float(ys[4 * j4 + 3]), __uint_as_float(yv[4 * j4 + 3])));
          }
        }
        const bool more = c + 1 < nchunks && build_m(c + 1);
        // stage the y tile as [t][p] and store it (the staging buffer's previous stores ended at the last barrier)
        const int pr = q * 32 + lane;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          *reinterpret_cast<uint16_t*>(smem + L::Y_OFF + (2 * j) * L::YLD + pr * 2) = static_cast<uint16_t>(yp[j]);
          *reinterpret_cast<uint16_t*>(smem + L::Y_OFF + (2 * j + 1) * L::YLD + pr * 2) =
              static_cast<uint16_t>(yp[j] >> 16);
        }
        asm volatile("bar.sync 2, 128;\n" ::: "memory");
        for (int i = tl; i < SQ * (SP / 8); i += 128) {
          const int t = i / (SP / 8), cc = i % (SP / 8);
          // 16-byte piece cc of the row: p 8 cc of the head, or p 8 (cc % 8) of head cc / 8
          if (t < qn)
            st16(P.out + static_cast<int64_t>(c0 + t) * P.o_t + (h + (HP == 1 ? 0 : cc / 8)) * P.o_h +
                     (HP == 1 ? cc : cc % 8) * 8,
                 *reinterpret_cast<const uint4*>(smem + L::Y_OFF + t * L::YLD + cc * 16));
        }
        asm volatile("bar.sync 2, 128;\n" ::: "memory");  // the y tile is reusable
        if (c + 1 < nchunks && !more) break;
      }
    }
  }

  // teardown: every MMA has completed (bounded) before TMEM is released
  mbar_drain(bar(B_DONE), 0);
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

template <typename ST, int N, int HP>
int launch_ssd_tc(const CUtensorMap& mx, const CUtensorMap& mb, const CUtensorMap& mc, const SsdTcParams& P, int nseq,
                  cudaStream_t s) {
  using L = TcSsdSmem<N, HP>;
  auto kern = ssd_prefill_tc_kernel<ST, N, HP>;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::DYN);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssd_prefill: smem attribute: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  cudaError_t e = mmp::launch(kern, dim3(P.nh / HP, nseq), dim3(STHR), L::DYN, s, nullptr, 0, mx, mb, mc, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssd_prefill: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_ssd_prefill");
}

}  // namespace

// The tensor-core path for head dim 128 with d_state 128 / 256, and head dim 64 with d_state 128 (two heads of one
// B/C group per CTA) with TMA-compatible strides; MMP_UNSUPPORTED otherwise (the caller then runs the mma.sync kernel).
int ssd_prefill_tc(const void* x, int64_t x_t, int64_t x_h, const void* dt, int64_t dt_t, int64_t dt_h, const float* A,
                   const float* D, const float* dt_bias, const void* B, int64_t B_t, int64_t B_g, const void* C,
                   int64_t C_t, int64_t C_g, void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                   const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init, void* out,
                   int64_t o_t, int64_t o_h, int nseq, int ntok, int nh, int p, int N, int ngroups, int lines, int* err,
                   cudaStream_t stream) {
  const bool two_heads = p == 64 && N == 128 && ngroups > 0 && nh % ngroups == 0 && (nh / ngroups) % 2 == 0;
  if ((p != SP && !two_heads) || (N != 128 && N != 256) || ntok <= 0 || nh > 65535 || nseq > 65535)
    return MMP_ERR_UNSUPPORTED;
  if (x_h % 8 || x_t % 8 || B_g % 8 || B_t % 8 || C_g % 8 || C_t % 8 || !aligned16(x) || !aligned16(B) ||
      !aligned16(C) || o_t % 8 || o_h % 8 || !aligned16(out) || s_p < N)
    return MMP_ERR_UNSUPPORTED;
  int rc = get_encoder();
  if (rc != MMP_OK) return rc;
  CUtensorMap mx, mb, mc;
  if ((rc = make_map3(&mx, x, p, nh, ntok, x_h, x_t)) || (rc = make_map3(&mb, B, N, ngroups, ntok, B_g, B_t)) ||
      (rc = make_map3(&mc, C, N, ngroups, ntok, C_g, C_t)))
    return rc;
  SsdTcParams P{static_cast<const bf16*>(dt), dt_t, dt_h, A, D, dt_bias, state, s_line, s_head, s_p,
                cu_seqlens, state_idx, has_init, static_cast<bf16*>(out), o_t, o_h, nh, ngroups, lines, err};
  const bool f32 = state_dtype == MMP_F32;
  if (two_heads)
    return f32 ? launch_ssd_tc<float, 128, 2>(mx, mb, mc, P, nseq, stream) : launch_ssd_tc<bf16, 128, 2>(mx, mb, mc, P, nseq, stream);
  if (N == 256) return f32 ? launch_ssd_tc<float, 256, 1>(mx, mb, mc, P, nseq, stream) : launch_ssd_tc<bf16, 256, 1>(mx, mb, mc, P, nseq, stream);
  return f32 ? launch_ssd_tc<float, 128, 1>(mx, mb, mc, P, nseq, stream) : launch_ssd_tc<bf16, 128, 1>(mx, mb, mc, P, nseq, stream);
}

}  // namespace mmp
