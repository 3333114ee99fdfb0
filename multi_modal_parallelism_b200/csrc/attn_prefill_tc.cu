// Causal GQA prefill attention over the paged KV cache on the 5th-generation tensor cores (tcgen05 / TMEM /
// TMA), head dim 128: the same operation as attn_prefill.cu (FlashAttention-2 varlen, causal, in the serving stack
// the reference measures). It is the default path for head dim 128; mmp_set_attn_prefill_tc(0) selects the mma.sync
// kernel instead, which also serves every shape this kernel does not.
//
// Query token j of sequence i sits at position ctx_start[i] + j and sees cache positions [0, ctx_start[i] + j]
// of that sequence. One CTA (10 warps) owns 128 query tokens of TWO query heads that read the same key/value
// head (a head pair; the last pair of a key/value head holds one head when the group size is odd), so every
// key/value tile it loads serves both, and each head has its own softmax warpgroup, so the two softmaxes share
// the SM's issue slots and hide each other's latencies while the tensor pipe alternates between the heads:
//   * warps 0-3 (head A) and 4-7 (head B), one query row per thread = one TMEM lane: load the head's Q tile with
//     plain 16-byte loads into the 128-byte-swizzled K-major operand layout, run the online softmax of every key
//     tile, write P (bf16) into TMEM over the scores it came from, and finally the epilogue;
//   * warp 8 gathers each tile of 128 keys page by page with 4-D TMA boxes [block_size keys x 64 dims] straight
//     from the paged K and V caches into a two-stage ring (pages past the sequence, or with a bad block id, are
//     requested at an out-of-range block coordinate and arrive as zeros);
//   * warp 9 (one thread) issues, for each head as soon as its inputs are ready, S_h(j) = Q_h K_j^T into the
//     head's score columns and O_h += P_h(j) V_j with P read from TMEM (the MMA's A operand) and V an MN-major
//     operand straight from its TMA boxes; S_h(j + 1) is issued only once O_h's update from P_h(j) has completed,
//     since it overwrites P_h(j)'s columns.
// The softmax keeps its running maximum lazily: O (in TMEM) and the row sum are rescaled only when a row's
// maximum grows by more than 2^8, so most tiles need no correction pass; P is rounded to bf16 as in the
// mma.sync kernel. Scores of keys a row may not see are replaced (not added to) by -inf, and value rows past
// the sequence's last key are zeroed (by head A's warps, before either head's last PV) so unwritten cache slots
// cannot turn 0 * x into NaN. Every mbarrier wait is bounded (tc_common.cuh); a CTA that runs out of budget flags
// the error word, stops issuing work, drains its copies and its MMAs, and frees TMEM.
#include <algorithm>

#include "mmp_common.cuh"
#include "tc_common.cuh"

namespace mmp {

static int g_attn_prefill_tc = 1;  // on by default; mmp_set_attn_prefill_tc(0) selects the mma.sync kernel

namespace {

constexpr int TQ = 128, TK = 128, THD = 128;
constexpr int TTHR = 320;  // warps 0-3 softmax head A, 4-7 head B, warp 8 copies, warp 9 MMAs

struct AttnTcSmem {
  static constexpr int Q_OFF = 0;                  // Q: 2 heads x 2 blocks [128 q][64 dims] (128 B rows, swizzled)
  static constexpr int K_OFF = Q_OFF + 65536;      // K ring: 2 stages x 2 blocks [128 keys][64 dims]
  static constexpr int V_OFF = K_OFF + 65536;      // V ring: same
  static constexpr int BAR_OFF = V_OFF + 65536;    // mbarriers (8 bytes each)
  static constexpr int NBAR = 16;
  static constexpr int FLAG_OFF = BAR_OFF + 8 * NBAR;
  static constexpr int USED = FLAG_OFF + 16;
  static constexpr int DYN = USED + 1024;          // + alignment of the base to 1024 bytes
  static constexpr int OST = THD * 2 + 16;         // output staging row (bytes): head A in the K ring, B in the V ring
};
static_assert(AttnTcSmem::DYN <= 232448, "shared memory per CTA");
static_assert(TQ * AttnTcSmem::OST <= 65536, "output staging of one head fits one ring");

// mbarrier slots (per head h: Q loaded, S ready, P written, O updated)
constexpr int B_Q = 0, B_K = 2, B_V = 4, B_EMPTY = 6, B_S = 8, B_P = 10, B_O = 12, B_DONE = 14;
// TMEM columns: head h's scores (and then its P, two bf16 per column, in the first 64) at T_S + 128 h, its output
// accumulator at T_O + 128 h
constexpr uint32_t T_S = 0, T_O = 256;

struct AttnTcParams {
  const bf16* q; int64_t q_t, q_h;
  const int32_t* block_table; int64_t bt_stride;
  const int32_t* cu_q; const int32_t* ctx_start;
  bf16* out; int64_t o_t, o_h;
  int nq, nkv, block_size, num_blocks, q_tiles;
  int pairs_per_kv;  // head pairs per key/value head: ceil((nq / nkv) / 2)
  int tok_inner;     // the cache maps list the token dimension before the head dimension (smaller stride first)
  float scale_log2;
  int* err;
};

__device__ __forceinline__ uint32_t swz128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }
__device__ __forceinline__ float ex2f(float x) {  // 2^x on the MUFU unit (ex2.approx.ftz; 2^-inf = 0)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];\n"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
// MN-major operand stored as [K rows][64 MN elements] blocks (128-byte swizzle), MN blocks `mn_block` bytes apart
__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr, uint32_t mn_block) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>((mn_block >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
constexpr uint32_t IDESC_B_MN_MAJOR = 1u << 16;
// MMA with the A operand in TMEM (K-major, two bf16 per 32-bit column, lane = row)
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
      ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate));
}

// grid (head pairs * nseq, q tiles): x = pair + pairs * sequence, pair = key/value head * pairs_per_kv + p; y counts
// query tiles from the last, so the CTAs with the longest key ranges are dispatched first and the short ones fill
// the tail
__global__ void __launch_bounds__(TTHR, 1) attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap mapK,
                                                                  const __grid_constant__ CUtensorMap mapV,
                                                                  const AttnTcParams P) {
  using L = AttnTcSmem;
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
  pdl_trigger();
  pdl_wait();
  const int npairs = P.nkv * P.pairs_per_kv;
  const int pair = blockIdx.x % npairs, seq = blockIdx.x / npairs;
  const int rep = P.nq / P.nkv;
  const int kh = pair / P.pairs_per_kv;
  const int head_a = kh * rep + 2 * (pair % P.pairs_per_kv);
  const int nh = head_a + 1 < (kh + 1) * rep ? 2 : 1;  // heads this CTA serves
  const int q0 = (P.q_tiles - 1 - static_cast<int>(blockIdx.y)) * TQ;
  const int qbase = P.cu_q[seq], qlen = P.cu_q[seq + 1] - qbase;
  if (q0 >= qlen) return;  // whole CTA: nothing initialised yet
  const int start = P.ctx_start[seq];
  const int rows = min(TQ, qlen - q0);
  const int total = start + qlen;           // keys of the sequence
  const int kend = start + q0 + rows;       // keys any row of this tile can see
  const int nkt = (kend + TK - 1) / TK;     // >= 1; only the last tile can reach past the sequence's last key
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sb = smem_addr(smem);
  auto bar = [&](int i) { return sb + L::BAR_OFF + 8 * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::FLAG_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::FLAG_OFF + 4);

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(B_Q + s), 128);
      mbar_init(bar(B_K + s), 1);
      mbar_init(bar(B_V + s), 1);
      mbar_init(bar(B_EMPTY + s), 1);
      mbar_init(bar(B_S + s), 1);
      mbar_init(bar(B_P + s), 128);
      mbar_init(bar(B_O + s), 1);
    }
    mbar_init(bar(B_DONE), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&mapK)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&mapV)) : "memory");
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
    // ---------------------------------------------------------------- copies: K and V tiles, page by page
    const int bs = P.block_size, nb = TK / bs;  // boxes per tile and 64-dim half (nb <= 16)
    const int32_t* btab = P.block_table + static_cast<int64_t>(seq) * P.bt_stride;
    int issued = 0;
    for (int j = 0; j < nkt; ++j) {
      const int s = j & 1;
      int go = 1;  // decided by lane 0 alone, so the whole warp leaves together
      if (lane == 0) {
        if (j >= 2) go = mbar_wait(bar(B_EMPTY + s), ((j >> 1) - 1) & 1, abort_flag, P.err) ? 1 : 0;
        if (*abort_flag) go = 0;
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      // this lane's page of the tile: a block coordinate, or one past the cache (zeros) for pages past the
      // sequence and for bad block ids (flagged)
      int blk = P.num_blocks;
      if (lane < nb) {
        const int tok0 = j * TK + lane * bs;
        if (tok0 < total) {
          const int col = tok0 / bs;
          const int b = col < P.bt_stride ? __ldg(btab + col) : -1;
          if (b >= 0 && b < P.num_blocks) blk = b;
          else flag_error(P.err, DEVERR_INDEX);
        }
      }
      if (lane == 0) mbar_expect_tx(bar(B_K + s), 2 * TK * 128);
      __syncwarp();
      const int cy = P.tok_inner ? 0 : kh, cz = P.tok_inner ? kh : 0;  // (token, head) in map order
      if (lane < nb) {
        const uint32_t dst = sb + L::K_OFF + s * 32768 + lane * bs * 128;
        tma_load_4d(dst, &mapK, bar(B_K + s), 0, cy, cz, blk);
        tma_load_4d(dst + 16384, &mapK, bar(B_K + s), 64, cy, cz, blk);
      }
      __syncwarp();
      if (lane == 0) mbar_expect_tx(bar(B_V + s), 2 * TK * 128);
      __syncwarp();
      if (lane < nb) {
        const uint32_t dst = sb + L::V_OFF + s * 32768 + lane * bs * 128;
        tma_load_4d(dst, &mapV, bar(B_V + s), 0, cy, cz, blk);
        tma_load_4d(dst + 16384, &mapV, bar(B_V + s), 64, cy, cz, blk);
      }
      issued = j + 1;
    }
    // copies in flight may still land after an abort: wait (bounded) for the last tile of each stage
    if (lane == 0) {
      for (int j = max(0, issued - 2); j < issued; ++j) {
        mbar_drain(bar(B_K + (j & 1)), (j >> 1) & 1);
        mbar_drain(bar(B_V + (j & 1)), (j >> 1) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMAs (one thread), head by head as ready
    if (lane == 0) {
      constexpr uint32_t id_s = umma_idesc_mn(TQ, TK);
      constexpr uint32_t id_o = umma_idesc_mn(TQ, THD) | IDESC_B_MN_MAJOR;
      auto issue_s = [&](int h, int j) {  // S_h(j) = Q_h K_j^T into head h's score columns
        const uint32_t kst = sb + L::K_OFF + (j & 1) * 32768;
#pragma unroll
        for (int kk = 0; kk < THD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16(tmem + T_S + h * TK, umma_desc(sb + L::Q_OFF + h * 32768 + off), umma_desc(kst + off), id_s,
                   kk != 0);
        }
        umma_commit(bar(B_S + h));
      };
      auto issue_pv = [&](int h, int j) {  // O_h += P_h V_j (K = keys; P from TMEM, 16 keys = 8 columns per step)
        const uint32_t vst = sb + L::V_OFF + (j & 1) * 32768;
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk)
          umma_f16_ts(tmem + T_O + h * THD, tmem + T_S + h * TK + kk * 8, desc_mn(vst + kk * 2048, 16384), id_o,
                      (j | kk) != 0);
        umma_commit(bar(B_O + h));  // PV_h(j) done: O_h stable, P_h's columns free
      };
      bool ok = mbar_wait(bar(B_Q), 0, abort_flag, P.err) && (nh < 2 || mbar_wait(bar(B_Q + 1), 0, abort_flag, P.err)) &&
                mbar_wait(bar(B_K), 0, abort_flag, P.err);
      if (ok) {
        tc_fence_after();
        for (int h = 0; h < nh; ++h) issue_s(h, 0);
      }
      int jp[2] = {0, nh > 1 ? 0 : nkt};  // next PV tile per head
      int js[2] = {1, nh > 1 ? 1 : nkt + 1};  // next S tile per head (S(0) issued)
      long long last = clock64();
      while (ok && (jp[0] < nkt || jp[1] < nkt)) {
        bool progressed = false;
        for (int h = 0; h < 2; ++h) {
          const int j = jp[h];
          if (j < nkt && js[h] == j + 1) {  // next: PV_h(j), once P_h(j) is written and V_j has landed (on the
                                            // last tile, head B's after head A's, whose warps zero the V tail)
            if (h == 1 && j == nkt - 1 && jp[0] <= j) continue;
            if (!mbar_try(bar(B_P + h), j & 1) || !mbar_try(bar(B_V + (j & 1)), (j >> 1) & 1)) continue;
            tc_fence_after();
            issue_pv(h, j);
            jp[h] = j + 1;
            if (jp[1 - h] > j) umma_commit(bar(B_EMPTY + (j & 1)));  // both heads' MMAs reading K_j, V_j issued
            progressed = true;
          } else if (js[h] < nkt && js[h] == j) {  // next: S_h(js), once PV_h(js - 1) is done and K_js has landed
            const int k = js[h];
            if (!mbar_try(bar(B_O + h), (k - 1) & 1) || !mbar_try(bar(B_K + (k & 1)), (k >> 1) & 1)) continue;
            tc_fence_after();
            issue_s(h, k);
            js[h] = k + 1;
            progressed = true;
          }
        }
        if (progressed) {
          last = clock64();
        } else if (*abort_flag) {
          ok = false;
        } else if (clock64() - last > WAIT_BUDGET_CYCLES) {
          *abort_flag = 1;
          flag_error(P.err, DEVERR_TIMEOUT);
          ok = false;
        }
      }
      umma_commit(bar(B_DONE));  // arrives once every MMA issued above has completed
    }
    __syncwarp();
  } else if (warp / 4 < nh) {
    // ---------------------------------------------------------------- warps 0-3 / 4-7: Q, softmax, epilogue
    const int h = warp / 4;
    const int r = tid & 127;  // query row = TMEM lane
    const uint32_t t_lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t t_s = t_lane + T_S + h * TK, t_o = t_lane + T_O + h * THD;
    // Q tile: thread i copies 16-byte chunk i % 16 of rows i / 16 + 8 n (rows past the sequence: zeros)
    for (int i = r; i < TQ * 16; i += 128) {
      const int qr = i >> 4, c = i & 15;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (qr < rows) v = ld16(P.q + static_cast<int64_t>(qbase + q0 + qr) * P.q_t + (head_a + h) * P.q_h + c * 8);
      *reinterpret_cast<uint4*>(smem + L::Q_OFF + h * 32768 + (c >> 3) * 16384 + swz128(qr, c & 7)) = v;
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic writes -> tensor core reads
    mbar_arrive(bar(B_Q + h));

    const int qpos = start + q0 + r;          // this row's position (rows >= `rows` are padding)
    const int vis = min(qpos, total - 1);     // last key this row sees
    const float sl = P.scale_log2;
    float m_used = -INFINITY;                 // running maximum in the exp2 domain (lazy)
    float lsum = 0.f;
    bool ok = true;
    int j = 0;
    for (; j < nkt; ++j) {
      ok = mbar_wait(bar(B_S + h), j & 1, abort_flag, P.err);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      uint32_t s[TK];
#pragma unroll
      for (int c = 0; c < TK / 16; ++c) tmem_ld16_nw(t_s + c * 16, s + c * 16);
      tmem_wait();
      const int k0 = j * TK;
      const int lim = vis - k0;  // keys k0 + c with c <= lim are visible
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < TK; ++c) {
        const float v = c <= lim ? __uint_as_float(s[c]) : -INFINITY;
        s[c] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
      const float m_new = mx * sl;
      const bool need = m_new > m_used + 8.f;  // false for -inf / NaN maxima
      if (__any_sync(0xffffffffu, need)) {
        const float alpha = need ? ex2f(m_used - m_new) : 1.f;  // 0 on the first visible tile
        if (need) {
          m_used = m_new;
          lsum *= alpha;
        }
        if (j > 0) {  // O holds PV(0 .. j-1), all complete (S(j) was issued after the last of them): rescale
#pragma unroll 1
          for (int c = 0; c < THD; c += 32) {
            uint32_t o[32];
            tmem_ld16_nw(t_o + c, o);
            tmem_ld16_nw(t_o + c + 16, o + 16);
            tmem_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st16(t_o + c, o);
            tmem_st16(t_o + c + 16, o + 16);
          }
        }
      }
      const float base = m_used == -INFINITY ? 0.f : m_used;
      float part = 0.f;
#pragma unroll
      for (int c = 0; c < TK; c += 2) {
        const float p0 = ex2f(fmaf(__uint_as_float(s[c]), sl, -base));
        const float p1 = ex2f(fmaf(__uint_as_float(s[c + 1]), sl, -base));
        part += p0 + p1;
        s[c / 2] = pack_bf16x2(p0, p1);  // P (bf16 pairs) in place: column c / 2 of the score columns
      }
      lsum += part;
      if (h == 0 && k0 + TK > total) {
        // value rows past the sequence's last key (the tail of its last page) may hold anything: zero them once
        // the tile has landed, before the PVs of either head read it
        ok = mbar_wait(bar(B_V + (j & 1)), (j >> 1) & 1, abort_flag, P.err);
        if (!(ok = __all_sync(0xffffffffu, ok))) break;
        if (r >= total - k0) {
          uint8_t* vrow = smem + L::V_OFF + (j & 1) * 32768 + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(vrow + 16384 + c * 16) = make_uint4(0, 0, 0, 0);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      }
#pragma unroll
      for (int c = 0; c < TK / 2; c += 16) tmem_st16(t_s + c, s + c);
      tmem_wait_st();
      tc_fence_before();  // the P and O writes precede the MMAs issued after the arrive
      mbar_arrive(bar(B_P + h));
    }
    // epilogue: once every MMA is done (the K / V rings are then idle), normalise O, stage bf16 rows in this
    // head's ring, store coalesced
    bool fin = ok && j == nkt && !*abort_flag;
    fin = fin && mbar_wait(bar(B_DONE), 0, abort_flag, P.err);
    fin = __all_sync(0xffffffffu, fin);
    if (fin) {
      tc_fence_after();
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
      uint8_t* orow = smem + (h ? L::V_OFF : L::K_OFF) + r * L::OST;
#pragma unroll 1
      for (int c = 0; c < THD; c += 32) {
        uint32_t o[32];
        tmem_ld16_nw(t_o + c, o);
        tmem_ld16_nw(t_o + c + 16, o + 16);
        tmem_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 8)
          *reinterpret_cast<uint4*>(orow + (c + e) * 2) = make_uint4(
              pack_bf16x2(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv),
              pack_bf16x2(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv),
              pack_bf16x2(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv),
              pack_bf16x2(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv));
      }
    }
    if (h == 0) asm volatile("bar.sync 1, 128;\n" ::: "memory");  // this head's four warps only
    else asm volatile("bar.sync 2, 128;\n" ::: "memory");
    if (!*abort_flag) {
      const uint8_t* stage = smem + (h ? L::V_OFF : L::K_OFF);
      for (int i = r; i < rows * (THD / 8); i += 128) {
        const int qr = i / (THD / 8), c = i % (THD / 8);
        st16(P.out + static_cast<int64_t>(qbase + q0 + qr) * P.o_t + (head_a + h) * P.o_h + c * 8,
             *reinterpret_cast<const uint4*>(stage + qr * L::OST + c * 16));
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

// 4-D tensor map over a paged cache [num_blocks][block_size][nkv][128] (bf16, strided): dimensions 128 dims,
// then token and head in order of increasing stride (tok_inner: token first), then block; the box (64 dims, a
// whole page of tokens, one head, one block) lands as block_size rows of 128 bytes either way
int make_cache_map(CUtensorMap* map, const void* base, int nkv, int block_size, int num_blocks, int64_t c_head,
                   int64_t c_tok, int64_t c_block, bool tok_inner) {
  const cuuint64_t bsz = static_cast<cuuint64_t>(block_size), nk = static_cast<cuuint64_t>(nkv);
  const cuuint64_t st = static_cast<cuuint64_t>(c_tok) * 2, sh = static_cast<cuuint64_t>(c_head) * 2;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(THD), tok_inner ? bsz : nk, tok_inner ? nk : bsz,
                        static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[3] = {tok_inner ? st : sh, tok_inner ? sh : st, static_cast<cuuint64_t>(c_block) * 2};
  cuuint32_t box[4] = {64, tok_inner ? static_cast<cuuint32_t>(block_size) : 1u,
                       tok_inner ? 1u : static_cast<cuuint32_t>(block_size), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {  // a layout the copy engine cannot describe: the caller runs the mma.sync kernel
    mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_paged_attn_prefill: cache tensor map not encodable (%d)", (int)r);
    return MMP_ERR_UNSUPPORTED;
  }
  return MMP_OK;
}

}  // namespace

// The tensor-core path when it is selected and the request fits it (head dim 128, a power-of-two page of 8 to
// 128 tokens, 16-byte aligned rows and output); MMP_ERR_UNSUPPORTED otherwise (the caller runs the mma.sync
// kernel). Arguments as mmp_paged_attn_prefill, already validated there.
int attn_prefill_tc(const void* q, int64_t q_t, int64_t q_h, const void* key_cache, const void* value_cache,
                    int64_t c_block, int64_t c_tok, int64_t c_head, const int32_t* block_table, int64_t bt_stride,
                    const int32_t* cu_q, const int32_t* ctx_start, void* out, int64_t o_t, int64_t o_h, int nseq,
                    int max_q_len, int nq, int nkv, int hd, int block_size, int num_blocks, float scale, int* err,
                    cudaStream_t stream) {
  if (!g_attn_prefill_tc) return MMP_ERR_UNSUPPORTED;
  if (hd != THD || block_size < 8 || block_size > TK || (block_size & (block_size - 1)) || o_t % 8 || o_h % 8 ||
      !aligned16(out) || nq % nkv || static_cast<int64_t>(nq) * nseq > 0x7fffffff)
    return MMP_ERR_UNSUPPORTED;
  const int q_tiles = (max_q_len + TQ - 1) / TQ;
  if (q_tiles > 65535) return MMP_ERR_UNSUPPORTED;
  int rc = get_encoder();
  if (rc != MMP_OK) return rc;
  const bool tok_inner = c_tok <= c_head;
  CUtensorMap mk, mv;
  if ((rc = make_cache_map(&mk, key_cache, nkv, block_size, num_blocks, c_head, c_tok, c_block, tok_inner)) ||
      (rc = make_cache_map(&mv, value_cache, nkv, block_size, num_blocks, c_head, c_tok, c_block, tok_inner)))
    return rc;
  const int pairs_per_kv = (nq / nkv + 1) / 2;
  AttnTcParams P{static_cast<const bf16*>(q), q_t, q_h, block_table, bt_stride, cu_q, ctx_start,
                 static_cast<bf16*>(out), o_t, o_h, nq, nkv, block_size, num_blocks, q_tiles, pairs_per_kv,
                 tok_inner ? 1 : 0, scale * 1.4426950408889634f, err};
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         AttnTcSmem::DYN);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_prefill: smem attribute: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  cudaError_t e = mmp::launch(attn_prefill_tc_kernel, dim3(nkv * pairs_per_kv * nseq, q_tiles), dim3(TTHR),
                              AttnTcSmem::DYN, stream, nullptr, 0, mk, mv, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_prefill: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_paged_attn_prefill");
}

}  // namespace mmp

extern "C" int mmp_set_attn_prefill_tc(int enable) {
  const int prev = mmp::g_attn_prefill_tc;
  mmp::g_attn_prefill_tc = enable ? 1 : 0;
  return prev;
}
