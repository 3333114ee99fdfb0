// Gated DeltaNet chunked prefill on the 5th-generation tensor cores (tcgen05 / TMEM / TMA), head dims 128 x 128.
// The algorithm and its parameters are those of mmp_gdn_prefill (gdn.cu); this file splits it into two passes so
// that the only serial part, the walk over a sequence's chunks, carries nothing but the state-dependent work.
//
// Per value head, for a 64-token chunk starting from state S (cum = running sum of the log decay g inside the
// chunk, gam_i = exp(cum_i), w_i = exp(cum_C - cum_i), K^ / Q^ the L2-normalised rows, Q^ also times dk^-1/2):
//   N_ij  = beta_i exp(cum_i - cum_j) k^_i.k^_j (j < i),   T = (I + N)^-1,   Qm_ij = exp(cum_i - cum_j) q^_i.k^_j (j <= i)
//   W     = T diag(beta gam) K^,   U0 = T diag(beta) V           (the chunk's WY form of the delta rule)
//   U^T   = U0^T - S W^T
//   O^T   = S (diag(gam) Q^)^T + U^T Qm^T
//   S'    = gam_C S + U^T diag(w) K^
// (the recurrence S_t = exp(g_t) S_{t-1} (I - beta_t k_t k_t^T) + beta_t v_t k_t^T unrolled over the chunk).
//
// Pass 1, gdn_chunk_prep_kernel: one CTA per (chunk, key head), every chunk of every sequence at once. The raw q
// and k rows arrive by TMA; one tcgen05.mma computes [K; Q] K^T (M = 128, N = 64, K = 128) into TMEM, and each
// warpgroup, for one value head of the key head, scales it by the row norms and the decays into N (fp32, shared
// memory) and Qm (bf16, to a workspace), then inverts I + N in fp32 on the CUDA cores (forward substitution, one
// column per thread, held in registers, the rows of N read as shared-memory broadcasts) and writes T (bf16) to the
// workspace. Nothing here depends on the state.
//
// Pass 2, gdn_walk_tc_kernel: one CTA per (value head, sequence) walks the chunks with S [dv = 128 lanes x dk = 128
// columns] fp32 resident in TMEM. Warp roles:
//   * warp 12: one thread streams q, k (key head), v (value head), T and Qm of each chunk through a three-stage
//     ring of 128-byte-swizzled TMA boxes; then the warp computes the chunk's gates (gam, beta, w, gam_C);
//   * warp 13: one thread issues the MMAs: X = S_bf W^T and O = S_bf (gam Q^)^T (A: the bf16 copy of S, read from
//     TMEM), S += (U w)_bf K^ and O += U_bf Qm^T (A: U from TMEM), and one chunk ahead W^T = K^^T (T beta gam)^T
//     and U0^T = V^T (T beta)^T (M = 128 over dk / dv, N = 64 tokens, K = 64 tokens);
//   * warps 0-3 (prep): normalise k in place (K^), q in place times gam (gam Q^), T -> T beta in place and
//     T beta gam into its own buffer; then move W^T out of TMEM into shared memory as the bf16 operand of X;
//   * warps 4-7 (state, one dv row per thread): the state pass (bf16 copy of S into TMEM, gam_C S back) and
//     U^T = U0^T - X into TMEM as bf16, plain and times w;
//   * warps 8-11 (output, one dv row per thread): O out of TMEM, the per-token RMS over the head's 128 values
//     (warp reduce-scatter + 4 partials), staged as token rows over the chunk's dead q / k boxes, gate silu(z)
//     (16-byte loads requested a chunk ahead) and bf16 stores as 16-byte pieces of rows; the stage returns to the
//     copy warp once the staging has been read.
// The state chain per chunk is the state pass, X, U and the state update; the W / U0 MMAs, their copy, the output
// and the loads run beside it, and the ring's recycling (load, operand preparation, output staging over the stage)
// sets the pace. Every mbarrier wait is bounded (wait_sleep, with the clock budget of tc_common.cuh); a CTA that
// runs out of budget flags the error word, leaves its state line untouched, drains its copies and MMAs and frees TMEM.
#include <algorithm>

#include "mmp_common.cuh"
#include "tc_common.cuh"

namespace mmp {
namespace {

constexpr int GC = 64;    // tokens per chunk
constexpr int GD = 128;   // dk == dv

struct GdnTcParams {
  const bf16* q; int64_t q_t, q_h;   // [T, nk, dk] post-conv, not normalised
  const bf16* k; int64_t k_t, k_h;
  const bf16* v; int64_t v_t, v_h;   // [T, nv, dv]
  const bf16* a; int64_t a_t;        // [T, nv] raw
  const bf16* b; int64_t b_t;
  const float* A_log; const float* dt_bias;
  const bf16* z; int64_t z_t, z_h;   // [T, nv, dv] or null
  const bf16* norm_w; float eps;     // [dv] or null
  float* state; int64_t s_line, s_head, s_row;
  const int32_t* cu_seqlens; const int32_t* state_idx; const int32_t* has_init;
  bf16* out; int64_t o_t, o_h;
  bf16* Tw; bf16* Qmw;               // workspace: [T, nv, 64] bf16 each (row i of the token's chunk matrix)
  int nseq, ntok, nk, nv, lines;
  int* err;
};

__device__ __forceinline__ float gdn_g(float a_raw, float dtb, float A_log, bool has_A) {
  return -(has_A ? __expf(A_log) : 1.f) * softplus(a_raw + dtb);
}

// Raw gate projections of one chunk for value head j, tokens 2 lane and 2 lane + 1, as bf16 bit patterns (nothing
// is computed from them here, so a load in flight does not hold the warp up until chunk_gates needs it).
__device__ __forceinline__ void gate_raw(const GdnTcParams& P, int64_t t0, int qn, int j, int lane, uint32_t (&ar)[2],
                                         uint32_t (&br)[2]) {
  const unsigned short* pa = reinterpret_cast<const unsigned short*>(P.a);
  const unsigned short* pb = reinterpret_cast<const unsigned short*>(P.b);
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int r = lane * 2 + e;
    ar[e] = r < qn ? __ldg(pa + (t0 + r) * P.a_t + j) : 0u;
    br[e] = r < qn ? __ldg(pb + (t0 + r) * P.b_t + j) : 0u;
  }
}

// Gates of one chunk from its raw projections (gate_raw): inclusive running sum of g (cum), beta (zero past qn),
// and the chunk total. Both passes call this, so their decays agree bit for bit.
__device__ __forceinline__ void chunk_gates(const GdnTcParams& P, const uint32_t (&ar)[2], const uint32_t (&br)[2],
                                            int qn, int j, int lane, float (&cum)[2], float (&beta)[2], float& total) {
  const bool has_A = P.A_log != nullptr;
  const float A_log = has_A ? P.A_log[j] : 0.f, dtb = P.dt_bias ? P.dt_bias[j] : 0.f;
  float gg[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const bool ok = lane * 2 + e < qn;
    gg[e] = ok ? gdn_g(__uint_as_float(ar[e] << 16), dtb, A_log, has_A) : 0.f;
    beta[e] = ok ? __fdividef(1.f, 1.f + __expf(-__uint_as_float(br[e] << 16))) : 0.f;
  }
  const float c1 = gg[0] + gg[1];
  float run = c1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float x = __shfl_up_sync(0xffffffffu, run, o);
    if (lane >= o) run += x;
  }
  total = __shfl_sync(0xffffffffu, run, 31);
  cum[0] = run - c1 + gg[0];
  cum[1] = run;
}

// The chunk `cid` of the flattened list (sequences in order, ceil(len / 64) chunks each): its sequence and first
// token; false when cid is past the last chunk. Every lane of the calling warp gets the same answer.
__device__ __forceinline__ bool locate_chunk(const int32_t* cu, int nseq, int cid, int lane, int& seq, int& c0, int& t_end) {
  int base = 0;
  for (int s0 = 0; s0 < nseq; s0 += 32) {
    const int s = s0 + lane;
    int n = 0;
    if (s < nseq) n = (cu[s + 1] - cu[s] + GC - 1) / GC;
    int run = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, run, o);
      if (lane >= o) run += x;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, s < nseq && cid < base + run);
    if (hit) {
      const int l = __ffs(hit) - 1;
      const int excl = __shfl_sync(0xffffffffu, base + run - n, l);
      seq = s0 + l;
      c0 = cu[seq] + (cid - excl) * GC;
      t_end = cu[seq + 1];
      return true;
    }
    base += __shfl_sync(0xffffffffu, run, 31);
  }
  return false;
}

__device__ __forceinline__ uint32_t swz128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Bounded wait whose threads sleep in the barrier (try_wait with a suspend-time hint: a suspended thread resumes
// when the phase completes) instead of spinning: a waiting warp leaves its issue slots to the working ones.
constexpr uint32_t WAIT_HINT_NS = 20000;
// Non-blocking test of a phase (test_wait never suspends)
__device__ __forceinline__ bool phase_done(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n.reg .pred p;\nmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait_sleep(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(bar), "r"(parity), "r"(WAIT_HINT_NS) : "memory");
    if (ok) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > WAIT_BUDGET_CYCLES) {
      *abort_flag = 1;
      flag_error(err, DEVERR_TIMEOUT);
      return false;
    }
  }
}

// UMMA descriptor of an MN-major operand stored as boxes [K rows][64 MN elements] (128-byte swizzle): 8-row K groups
// 1024 bytes apart, 64-element MN blocks `mn_block` bytes apart
__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr, uint32_t mn_block) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>((mn_block >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
constexpr uint32_t A_MN = 1u << 15, B_MN = 1u << 16;

// MMA whose A operand is in TMEM (K-major, two bf16 per 32-bit column, lane = row)
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
      ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void arrive1(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  tmem_ld16_nw(taddr, r);
  tmem_ld16_nw(taddr + 16, r + 16);
}
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t* r) {
  tmem_ld32(taddr, r);
  tmem_ld32(taddr + 32, r + 32);
}
__device__ __forceinline__ bool and_bar(int id, int nthreads, bool v) {
  int r;
  asm volatile("{\n.reg .pred p, q;\nsetp.ne.s32 p, %1, 0;\nbar.red.and.pred q, %2, %3, p;\nselp.s32 %0, 1, 0, q;\n}\n"
               : "=r"(r) : "r"(v ? 1 : 0), "r"(id), "r"(nthreads) : "memory");
  return r != 0;
}

// ============================================================================================ pass 1
constexpr int PTHR = 256;  // two warpgroups, one value head each at a time
constexpr int NLD = 68;    // fp32 row stride of N and T (float4 rows without bank conflicts)

struct PrepSmem {
  static constexpr int QK = 0;            // k-block kb at kb * 16384: K rows 0-63, then Q rows 0-63 (128 B each)
  static constexpr int RK = 32768;        // [64] |k|^-1, then [64] dk^-1/2 |q|^-1
  static constexpr int WG = RK + 512;     // per warpgroup:
  static constexpr int CUM = 0, BETA = 256, N = 512, TF = N + 64 * NLD * 4;
  static constexpr int WG_BYTES = TF + 64 * NLD * 4;
  static constexpr int BAR = WG + 2 * WG_BYTES;
  static constexpr int USED = BAR + 32;
  static constexpr int DYN = USED + 1024;
};
static_assert(PrepSmem::WG_BYTES % 16 == 0 && PrepSmem::DYN * 2 <= 232448, "two chunk CTAs per SM");

__global__ void __launch_bounds__(PTHR, 2) gdn_chunk_prep_kernel(const __grid_constant__ CUtensorMap mapQ,
                                                                 const __grid_constant__ CUtensorMap mapK,
                                                                 const GdnTcParams P) {
  using L = PrepSmem;
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = dsmem + ((1024u - (smem_addr(dsmem) & 1023u)) & 1023u);  // 1024-aligned, still a shared pointer
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kh = blockIdx.y;
  int seq = 0, c0 = 0, t_end = 0;
  if (!locate_chunk(P.cu_seqlens, P.nseq, blockIdx.x, lane, seq, c0, t_end)) return;  // the same in every warp
  const int qn = min(GC, t_end - c0);
  const uint32_t sb = smem_addr(smem);
  const uint32_t bar_ld = sb + L::BAR, bar_mma = sb + L::BAR + 8;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L::BAR + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::BAR + 20);
  if (tid == 0) {
    mbar_init(bar_ld, 1);
    mbar_init(bar_mma, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&mapQ)) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&mapK)) : "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 64;\n" ::"r"(smem_addr(tslot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  bool issued = false;
  if (tid == 0) {
    mbar_expect_tx(bar_ld, 32768);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      tma_load_3d(sb + L::QK + kb * 16384, &mapK, bar_ld, kb * 64, kh, c0);
      tma_load_3d(sb + L::QK + kb * 16384 + 8192, &mapQ, bar_ld, kb * 64, kh, c0);
    }
  }
  // the first value head's raw gates, requested before the wait on q / k (warp 0 of each warpgroup)
  const int rheads = P.nv / P.nk;
  uint32_t g_ar[2] = {0u, 0u}, g_br[2] = {0u, 0u};
  if ((warp & 3) == 0 && (warp >> 2) < rheads) gate_raw(P, c0, qn, kh * rheads + (warp >> 2), lane, g_ar, g_br);
  bool ok = wait_sleep(bar_ld, 0, abort_flag, P.err);
  if (tid == 0 && ok) {
    // D = [K; Q] K^T: M = 128 (rows of K, then of Q), N = 64 (rows of K), K = 128 (two 64-wide k-blocks)
    tc_fence_after();
    constexpr uint32_t idesc = umma_idesc_mn(128, 64);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_f16(tmem, umma_desc(sb + L::QK + kb * 16384 + kk * 32), umma_desc(sb + L::QK + kb * 16384 + kk * 32),
                 idesc, (kb | kk) != 0);
    umma_commit(bar_mma);
    issued = true;
  }
  float* rk = reinterpret_cast<float*>(smem + L::RK);
  float* rq = rk + 64;
  if (ok) {
    // row norms from the raw bf16 rows: two threads per row (one k-block each)
    const int row = tid >> 1, kb = tid & 1;
    const uint8_t* base = smem + L::QK + kb * 16384 + (row >= 64 ? 8192 : 0);
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 w = *reinterpret_cast<const uint4*>(base + swz128(row & 63, c));
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(ws[e]);
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    if (kb == 0) {
      if (row < 64) rk[row] = rsqrtf(ss + 1e-6f);
      else rq[row - 64] = rsqrtf(ss + 1e-6f) * rsqrtf(static_cast<float>(GD));
    }
  }
  __syncthreads();
  ok = ok && wait_sleep(bar_mma, 0, abort_flag, P.err);
  ok = __syncthreads_and(ok);
  if (ok) {
    tc_fence_after();
    const int wg = warp >> 2, u = tid & 127, wq = warp & 3;
    const int bar_id = 1 + wg;
    uint8_t* wgs = smem + L::WG + wg * L::WG_BYTES;
    float* sCum = reinterpret_cast<float*>(wgs + L::CUM);
    float* sBeta = reinterpret_cast<float*>(wgs + L::BETA);
    float* sN = reinterpret_cast<float*>(wgs + L::N);
    float* sTf = reinterpret_cast<float*>(wgs + L::TF);
    for (int jj = wg; jj < rheads; jj += 2) {
      const int j = kh * rheads + jj;
      if (wq == 0) {
        if (jj != wg) gate_raw(P, c0, qn, j, lane, g_ar, g_br);
        float cum[2], beta[2], tot;
        chunk_gates(P, g_ar, g_br, qn, j, lane, cum, beta, tot);
        *reinterpret_cast<float2*>(sCum + 2 * lane) = make_float2(cum[0], cum[1]);
        *reinterpret_cast<float2*>(sBeta + 2 * lane) = make_float2(beta[0], beta[1]);
      }
      asm volatile("bar.sync %0, 128;\n" ::"r"(bar_id) : "memory");
      // row u of D: rows 0-63 give N (fp32, shared memory), rows 64-127 give Qm (bf16, straight to the workspace)
      uint32_t d[64];
      tmem_ld64(tmem + (static_cast<uint32_t>(wq * 32) << 16), d);
      tmem_wait();
      if (u < 64) {
        const int i = u;
        const float ci = sCum[i], bi = sBeta[i] * rk[i];
        const bool vi = i < qn;
#pragma unroll
        for (int c4 = 0; c4 < 16; ++c4) {
          float n[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int jx = c4 * 4 + e;
            n[e] = (vi && jx < i) ? bi * __expf(ci - sCum[jx]) * rk[jx] * __uint_as_float(d[jx]) : 0.f;
          }
          *reinterpret_cast<float4*>(sN + i * NLD + c4 * 4) = make_float4(n[0], n[1], n[2], n[3]);
        }
        // T = (I + N)^-1 by forward substitution, one column per thread (column u), in registers: t_i = -sum_{m < i}
        // N_im t_m below the diagonal, with the rows of N read as broadcasts (every thread reads the same row)
        asm volatile("bar.sync %0, 64;\n" ::"r"(bar_id + 2) : "memory");
        float t[GC];
#pragma unroll
        for (int ii = 0; ii < GC; ++ii) {
          float acc = 0.f;
#pragma unroll
          for (int m4 = 0; m4 < (ii + 3) / 4; ++m4) {  // N_im = 0 for m >= i
            const float4 nv4 = *reinterpret_cast<const float4*>(sN + ii * NLD + 4 * m4);
            acc = fmaf(nv4.x, t[4 * m4], acc);
            if (4 * m4 + 1 < ii) acc = fmaf(nv4.y, t[4 * m4 + 1], acc);
            if (4 * m4 + 2 < ii) acc = fmaf(nv4.z, t[4 * m4 + 2], acc);
            if (4 * m4 + 3 < ii) acc = fmaf(nv4.w, t[4 * m4 + 3], acc);
          }
          t[ii] = ii == u ? 1.f : (ii < u ? 0.f : -acc);
        }
        // column u into T's rows (a warp writes 32 consecutive floats of each row), then each thread one row
#pragma unroll
        for (int ii = 0; ii < GC; ++ii) sTf[ii * NLD + u] = t[ii];
        asm volatile("bar.sync %0, 64;\n" ::"r"(bar_id + 2) : "memory");
        if (u < qn) {
          bf16* dst = P.Tw + (static_cast<int64_t>(c0 + i) * P.nv + j) * GC;
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            const float4 x0 = *reinterpret_cast<const float4*>(sTf + i * NLD + c8 * 8);
            const float4 x1 = *reinterpret_cast<const float4*>(sTf + i * NLD + c8 * 8 + 4);
            st16(dst + c8 * 8, make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w), pack_bf16x2(x1.x, x1.y),
                                          pack_bf16x2(x1.z, x1.w)));
          }
        }
      } else {
        const int i = u - 64;
        if (i < qn) {
          const float ci = sCum[i], si = rq[i];
          bf16* dst = P.Qmw + (static_cast<int64_t>(c0 + i) * P.nv + j) * GC;
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            float m[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int jx = c8 * 8 + e;
              m[e] = jx <= i ? __expf(ci - sCum[jx]) * si * rk[jx] * __uint_as_float(d[jx]) : 0.f;
            }
            st16(dst + c8 * 8, make_uint4(pack_bf16x2(m[0], m[1]), pack_bf16x2(m[2], m[3]), pack_bf16x2(m[4], m[5]),
                                          pack_bf16x2(m[6], m[7])));
          }
        }
      }
      asm volatile("bar.sync %0, 128;\n" ::"r"(bar_id) : "memory");  // buffers are rewritten for the next head
    }
  }
  // teardown: copies and the MMA in flight land before the CTA's memory goes away
  if (tid == 0) {
    mbar_drain(bar_ld, 0);
    if (issued) mbar_drain(bar_mma, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 64;\n" ::"r"(tmem));
  }
}

// ============================================================================================ pass 2
constexpr int WTHR = 448;  // warps 0-3 prep, 4-7 state, 8-11 output, 12 copies + gates, 13 MMAs

struct WalkSmem {
  static constexpr int STAGE = 65536;  // one chunk: q, k, v (two 64-wide boxes each), T, Qm (one box each)
  static constexpr int Q = 0, K = 16384, V = 32768, T = 49152, QM = 57344;
  static constexpr int NST = 3;
  static constexpr int TBG = NST * STAGE;   // T diag(beta gam) [64 i][64 j] bf16, K-major
  static constexpr int W = TBG + 8192;      // W^T as [128 d rows][64 i] bf16 (MN-major operand of X)
  static constexpr int GATE = W + 16384;    // ring of 4: gam[64], beta[64], w[64], gam_C
  static constexpr int GATE_BYTES = 3 * 256 + 16;
  static constexpr int PART = GATE + 4 * GATE_BYTES;  // [2][4][64] fp32 per-warp sums of squares of O
  static constexpr int BAR = PART + 2 * 4 * 64 * 4;
  static constexpr int NBAR = 20;
  static constexpr int USED = BAR + 8 * NBAR + 16;
  static constexpr int DYN = USED + 1024;
};
static_assert(WalkSmem::DYN <= 232448, "shared memory per CTA");

// TMEM columns: S fp32 [128], its bf16 copy [64], X [64], O [64], U bf16 [32], U w bf16 [32], W^T [64], U0^T [64]
struct WalkTmem {
  static constexpr uint32_t S = 0, SBF = 128, X = 192, O = 256, UBF = 320, UWBF = 352, WT = 384, U0T = 448;
};
static_assert(WalkTmem::U0T + 64 == 512, "TMEM columns");

// mbarriers (per chunk c, phase c & 1 unless noted; FULL / EMPTY per ring stage, phase (c / 3) & 1; GATES ring of
// four, phase (c / 4) & 1)
constexpr int WB_FULL = 0, WB_EMPTY = 3, WB_GATES = 6, WB_PREP = 10, WB_WU = 11, WB_WREADY = 12, WB_SP = 13,
              WB_XDONE = 14, WB_OFREE = 15, WB_UREADY = 16, WB_SDONE = 17, WB_ODONE = 18, WB_DONE = 19;

__global__ void __launch_bounds__(WTHR, 1) gdn_walk_tc_kernel(const __grid_constant__ CUtensorMap mapQ,
                                                              const __grid_constant__ CUtensorMap mapK,
                                                              const __grid_constant__ CUtensorMap mapV,
                                                              const __grid_constant__ CUtensorMap mapT,
                                                              const __grid_constant__ CUtensorMap mapQm,
                                                              const GdnTcParams P) {
  using L = WalkSmem;
  using TM = WalkTmem;
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = dsmem + ((1024u - (smem_addr(dsmem) & 1023u)) & 1023u);  // 1024-aligned, still a shared pointer
  pdl_trigger();
  pdl_wait();
  const uint32_t sb = smem_addr(smem);
  const int j = blockIdx.x, seq = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t_begin = P.cu_seqlens[seq], t_end = P.cu_seqlens[seq + 1];
  const int line = P.state_idx[seq];
  if (line < 0 || line >= P.lines) {
    if (tid == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const int nchunks = (t_end - t_begin + GC - 1) / GC;
  const int kh = j / (P.nv / P.nk);
  auto bar = [&](int i) { return sb + L::BAR + 8 * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::BAR + 8 * L::NBAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR + 8 * L::NBAR + 4);
  auto gates = [&](int c) { return reinterpret_cast<float*>(smem + L::GATE + (c & 3) * L::GATE_BYTES); };
  float* gstate = P.state + line * P.s_line + j * P.s_head;

  if (tid == 0) {
    for (int s = 0; s < L::NST; ++s) {
      mbar_init(bar(WB_FULL + s), 1);
      mbar_init(bar(WB_EMPTY + s), 2);  // the MMAs reading the stage, and the output group's staging over it
    }
    for (int i = 0; i < 4; ++i) mbar_init(bar(WB_GATES + i), 32);
    mbar_init(bar(WB_PREP), 128);
    mbar_init(bar(WB_WU), 1);
    mbar_init(bar(WB_WREADY), 128);
    mbar_init(bar(WB_SP), 128);
    mbar_init(bar(WB_XDONE), 1);
    mbar_init(bar(WB_OFREE), 128);
    mbar_init(bar(WB_UREADY), 128);
    mbar_init(bar(WB_SDONE), 1);
    mbar_init(bar(WB_ODONE), 1);
    mbar_init(bar(WB_DONE), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    const CUtensorMap* maps[5] = {&mapQ, &mapK, &mapV, &mapT, &mapQm};
    for (int m = 0; m < 5; ++m)
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(maps[m])) : "memory");
  }
  if (warp == 13) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(smem_addr(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);  // this warp's TMEM lanes

  if (warp == 12) {
    // ------------------------------------------------------------------ copies (one thread), then the gates (warp)
    int issued = 0;
    uint32_t ar[2], br[2];  // raw gates of the chunk about to be loaded, requested a chunk ahead
    if (nchunks > 0) gate_raw(P, t_begin, min(GC, t_end - t_begin), j, lane, ar, br);
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % L::NST;
      const int c0 = t_begin + c * GC;
      int go = 1;
      if (lane == 0) {
        if (c >= L::NST && !wait_sleep(bar(WB_EMPTY + s), ((c / L::NST) - 1) & 1, abort_flag, P.err)) go = 0;
        if (*abort_flag) go = 0;
        if (go) {
          const uint32_t st = sb + s * L::STAGE, full = bar(WB_FULL + s);
          mbar_expect_tx(full, L::STAGE);
#pragma unroll
          for (int kb = 0; kb < 2; ++kb) {
            tma_load_3d(st + L::Q + kb * 8192, &mapQ, full, kb * 64, kh, c0);
            tma_load_3d(st + L::K + kb * 8192, &mapK, full, kb * 64, kh, c0);
            tma_load_3d(st + L::V + kb * 8192, &mapV, full, kb * 64, j, c0);
          }
          tma_load_3d(st + L::T, &mapT, full, 0, j, c0);
          tma_load_3d(st + L::QM, &mapQm, full, 0, j, c0);
          if (c + L::NST < nchunks) {  // the chunk that reuses this stage, into L2
            const int cn = c0 + L::NST * GC;
#pragma unroll
            for (int kb = 0; kb < 2; ++kb) {
              tma_prefetch_3d(&mapQ, kb * 64, kh, cn);
              tma_prefetch_3d(&mapK, kb * 64, kh, cn);
              tma_prefetch_3d(&mapV, kb * 64, j, cn);
            }
            tma_prefetch_3d(&mapT, 0, j, cn);
            tma_prefetch_3d(&mapQm, 0, j, cn);
          }
          issued = c + 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      const int qn = min(GC, t_end - c0);
      float cum[2], beta[2], tot;
      chunk_gates(P, ar, br, qn, j, lane, cum, beta, tot);
      if (c + 1 < nchunks) gate_raw(P, c0 + GC, min(GC, t_end - c0 - GC), j, lane, ar, br);
      float* g = gates(c);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = 2 * lane + e;
        g[r] = r < qn ? __expf(cum[e]) : 0.f;
        g[64 + r] = beta[e];
        g[128 + r] = r < qn ? __expf(tot - cum[e]) : 0.f;
      }
      if (lane == 0) g[192] = __expf(tot);
      arrive1(bar(WB_GATES + (c & 3)));
    }
    // copies in flight may still land after an abort: wait (bounded) for the last chunk of each stage
    if (lane == 0)
      for (int c = max(0, issued - L::NST); c < issued; ++c) mbar_drain(bar(WB_FULL + c % L::NST), (c / L::NST) & 1);
    __syncwarp();
  } else if (warp == 13) {
    // ------------------------------------------------------------------ MMAs (one thread)
    if (lane == 0) {
      constexpr uint32_t id_x = umma_idesc_mn(128, 64) | B_MN;   // X = S_bf W^T        (B: W^T rows, MN-major)
      constexpr uint32_t id_o = umma_idesc_mn(128, 64);          // O = S_bf (gam Q)^T  (B: K-major rows of Q)
      constexpr uint32_t id_s = umma_idesc_mn(128, 128) | B_MN;  // S += (U w) K^       (B: K rows, MN-major)
      constexpr uint32_t id_q = umma_idesc_mn(128, 64);          // O += U Qm^T         (B: K-major rows of Qm)
      constexpr uint32_t id_w = umma_idesc_mn(128, 64) | A_MN;   // W^T, U0^T           (A: K / V rows, MN-major)
      auto stage = [&](int c) { return sb + (c % L::NST) * L::STAGE; };
      auto ready = [&](int c) {  // chunk c prepared by warps 0-3 and its copies landed
        return wait_sleep(bar(WB_PREP), c & 1, abort_flag, P.err) &&
               wait_sleep(bar(WB_FULL + c % L::NST), (c / L::NST) & 1, abort_flag, P.err);
      };
      auto issue_wu = [&](int c) {  // W^T = K^^T (T beta gam)^T, U0^T = V^T (T beta)^T (K = 64 tokens)
        const uint32_t st = stage(c);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem + TM::WT, desc_mn(st + L::K + kk * 2048, 8192), umma_desc(sb + L::TBG + kk * 32), id_w, kk != 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem + TM::U0T, desc_mn(st + L::V + kk * 2048, 8192), umma_desc(st + L::T + kk * 32), id_w, kk != 0);
        umma_commit(bar(WB_WU));
      };
      bool ok = nchunks > 0 && ready(0);
      if (ok) {
        tc_fence_after();
        issue_wu(0);
      }
      for (int c = 0; ok && c < nchunks; ++c) {
        const uint32_t par = c & 1, st = stage(c);
        // W(c) in shared memory and the state pass done: X = S_bf W^T (K = 128 over d)
        if (!(ok = wait_sleep(bar(WB_WREADY), par, abort_flag, P.err) && wait_sleep(bar(WB_SP), par, abort_flag, P.err)))
          break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ts(tmem + TM::X, tmem + TM::SBF + kk * 8, desc_mn(sb + L::W + kk * 2048, 8192), id_x, kk != 0);
        umma_commit(bar(WB_XDONE));
        // O = S_bf (gam Q^)^T, once the previous O is read out
        if (c > 0 && !(ok = wait_sleep(bar(WB_OFREE), par ^ 1, abort_flag, P.err))) break;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tmem + TM::O, tmem + TM::SBF + kb * 32 + kk * 8, umma_desc(st + L::Q + kb * 8192 + kk * 32), id_o,
                   (kb | kk) != 0);
        // U in TMEM: S += (U w)_bf K^ (K = 64 tokens)
        if (!(ok = wait_sleep(bar(WB_UREADY), par, abort_flag, P.err))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ts(tmem + TM::S, tmem + TM::UWBF + kk * 8, desc_mn(st + L::K + kk * 2048, 8192), id_s, 1);
        umma_commit(bar(WB_SDONE));
        // the next chunk's W^T / U0^T ahead of O += U Qm^T when it is prepared already (U0^T and W^T are read out)
        bool wu = false;
        if (c + 1 < nchunks && phase_done(bar(WB_PREP), (c + 1) & 1) &&
            phase_done(bar(WB_FULL + (c + 1) % L::NST), ((c + 1) / L::NST) & 1)) {
          tc_fence_after();
          issue_wu(c + 1);
          wu = true;
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ts(tmem + TM::O, tmem + TM::UBF + kk * 8, umma_desc(st + L::QM + kk * 32), id_q, 1);
        umma_commit(bar(WB_ODONE));
        umma_commit(bar(WB_EMPTY + c % L::NST));  // every MMA reading this stage has been issued
        if (c + 1 < nchunks && !wu) {
          if (!(ok = ready(c + 1))) break;
          tc_fence_after();
          issue_wu(c + 1);
        }
      }
      umma_commit(bar(WB_DONE));  // arrives once every MMA issued above has completed
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------------ warps 0-3: operands of each chunk, W^T
    const int u = tid;
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % L::NST;
      bool ok = wait_sleep(bar(WB_FULL + s), (c / L::NST) & 1, abort_flag, P.err) &&
                wait_sleep(bar(WB_GATES + (c & 3)), (c >> 2) & 1, abort_flag, P.err);
      if (!__all_sync(0xffffffffu, ok)) break;
      uint8_t* st = smem + s * L::STAGE;
      const float* g = gates(c);
      {
        // q and k rows in place, two threads per row (one 64-wide box each): K^ = k / |k|, gam Q^ = gam q / (|q| sqrt(dk))
        const int row = u >> 1, kb = u & 1;
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          uint8_t* base = st + (m == 0 ? L::K : L::Q) + kb * 8192;
          uint4 w[8];
          float sq[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial sums
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) w[ch] = *reinterpret_cast<const uint4*>(base + swz128(row, ch));
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const uint32_t ws[4] = {w[ch].x, w[ch].y, w[ch].z, w[ch].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = unpack_bf16x2(ws[e]);
              sq[e] = fmaf(f.x, f.x, fmaf(f.y, f.y, sq[e]));
            }
          }
          float ss = (sq[0] + sq[1]) + (sq[2] + sq[3]);
          ss += __shfl_xor_sync(0xffffffffu, ss, 1);
          const float sc = m == 0 ? rsqrtf(ss + 1e-6f) : rsqrtf(ss + 1e-6f) * rsqrtf(static_cast<float>(GD)) * g[row];
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const uint32_t ws[4] = {w[ch].x, w[ch].y, w[ch].z, w[ch].w};
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = unpack_bf16x2(ws[e]);
              o[e] = pack_bf16x2(f.x * sc, f.y * sc);
            }
            *reinterpret_cast<uint4*>(base + swz128(row, ch)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        // T beta in place and T beta gam into its buffer: thread = (row, half of the 64 columns)
        const float* gb = g + 64;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int ch = (u & 1) * 4 + cc;
          uint8_t* tp = st + L::T + swz128(row, ch);
          const uint4 t = *reinterpret_cast<const uint4*>(tp);
          const uint32_t ts[4] = {t.x, t.y, t.z, t.w};
          uint32_t ob[4], og[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int jx = ch * 8 + 2 * e;
            const float2 f = unpack_bf16x2(ts[e]);
            const float b0 = gb[jx], b1 = gb[jx + 1];
            ob[e] = pack_bf16x2(f.x * b0, f.y * b1);
            og[e] = pack_bf16x2(f.x * b0 * g[jx], f.y * b1 * g[jx + 1]);
          }
          *reinterpret_cast<uint4*>(tp) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
          *reinterpret_cast<uint4*>(smem + L::TBG + swz128(row, ch)) = make_uint4(og[0], og[1], og[2], og[3]);
        }
      }
      proxy_fence();  // generic shared-memory writes -> tensor-core reads
      arrive1(bar(WB_PREP));
      // W^T(c) out of TMEM (lane d) into the X operand: row d of [128 d][64 i] bf16
      ok = wait_sleep(bar(WB_WU), c & 1, abort_flag, P.err);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      uint32_t r[64];
      tmem_ld64(t_lane + TM::WT, r);
      tmem_wait();
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          o[e] = pack_bf16x2(__uint_as_float(r[ch * 8 + 2 * e]), __uint_as_float(r[ch * 8 + 2 * e + 1]));
        *reinterpret_cast<uint4*>(smem + L::W + swz128(u, ch)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      tc_fence_before();
      proxy_fence();
      arrive1(bar(WB_WREADY));
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------------ warps 4-7: the state, U
    const int u = tid - 128;  // dv row = TMEM lane
    const bool init = P.has_init && P.has_init[seq];
#pragma unroll 1
    for (int cn = 0; cn < GD; cn += 16) {
      uint32_t r[16];
      float4 f[4] = {};
      if (init)
#pragma unroll
        for (int e = 0; e < 4; ++e) f[e] = *reinterpret_cast<const float4*>(gstate + u * P.s_row + cn + 4 * e);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        r[4 * e] = __float_as_uint(f[e].x);
        r[4 * e + 1] = __float_as_uint(f[e].y);
        r[4 * e + 2] = __float_as_uint(f[e].z);
        r[4 * e + 3] = __float_as_uint(f[e].w);
      }
      tmem_st16(t_lane + TM::S + cn, r);
    }
    tmem_wait_st();
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      const uint32_t par = c & 1;
      const int qn = min(GC, t_end - t_begin - c * GC);
      if (c > 0) ok = wait_sleep(bar(WB_SDONE), par ^ 1, abort_flag, P.err);
      ok = ok && wait_sleep(bar(WB_GATES + (c & 3)), (c >> 2) & 1, abort_flag, P.err);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      const float* g = gates(c);
      const float dec = g[192];
      // the state pass: bf16 copy of the chunk's incoming state, gam_C S back (the update accumulates on it)
#pragma unroll 1
      for (int cn = 0; cn < GD; cn += 64) {
        uint32_t r[64], b[32];
        tmem_ld64(t_lane + TM::S + cn, r);
        tmem_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) b[e] = pack_bf16x2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
#pragma unroll
        for (int e = 0; e < 64; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * dec);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) tmem_st16(t_lane + TM::S + cn + 16 * k4, r + 16 * k4);
        tmem_st16(t_lane + TM::SBF + cn / 2, b);
        tmem_st16(t_lane + TM::SBF + cn / 2 + 16, b + 16);
      }
      tmem_wait_st();
      tc_fence_before();
      arrive1(bar(WB_SP));
      // U^T = U0^T - X (zero past the sequence end), as bf16 plain and times w
      ok = wait_sleep(bar(WB_XDONE), par, abort_flag, P.err);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      const float* w = g + 128;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t x[32], y[32], ub[16], uw[16];
        tmem_ld32(t_lane + TM::X + 32 * h, x);
        tmem_ld32(t_lane + TM::U0T + 32 * h, y);
        tmem_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int i0 = 32 * h + 2 * e;
          const float u0 = i0 < qn ? __uint_as_float(y[2 * e]) - __uint_as_float(x[2 * e]) : 0.f;
          const float u1 = i0 + 1 < qn ? __uint_as_float(y[2 * e + 1]) - __uint_as_float(x[2 * e + 1]) : 0.f;
          ub[e] = pack_bf16x2(u0, u1);
          uw[e] = pack_bf16x2(u0 * w[i0], u1 * w[i0 + 1]);
        }
        tmem_st16(t_lane + TM::UBF + 16 * h, ub);
        tmem_st16(t_lane + TM::UWBF + 16 * h, uw);
      }
      tmem_wait_st();
      tc_fence_before();
      arrive1(bar(WB_UREADY));
    }
    // final state -> the sequence's line (skipped after an abort: the line keeps its old value)
    if (ok && nchunks > 0) ok = wait_sleep(bar(WB_SDONE), (nchunks - 1) & 1, abort_flag, P.err);
    ok = __all_sync(0xffffffffu, ok) && !*abort_flag;
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int cn = 0; cn < GD; cn += 16) {
        uint32_t r[16];
        tmem_ld16_nw(t_lane + TM::S + cn, r);
        tmem_wait();
#pragma unroll
        for (int e = 0; e < 4; ++e)
          *reinterpret_cast<float4*>(gstate + u * P.s_row + cn + 4 * e) =
              make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]), __uint_as_float(r[4 * e + 2]),
                          __uint_as_float(r[4 * e + 3]));
      }
    }
  } else {
    // ------------------------------------------------------------------ warps 8-11: output rows
    // O (lane v, column i) times 1 / RMS and the norm weight is staged as fp32 [64 i][128 v] over the chunk's q / k
    // boxes (their last readers, the O1 and state MMAs, completed before O2), then each thread takes 16-byte pieces of
    // token rows: times silu(z) from coalesced 16-byte loads (requested a chunk ahead), bf16, coalesced 16-byte
    // stores. The stage is released to the copy warp (its second EMPTY arrival) once the staging has been read.
    const int u = tid - 256;  // dv row = TMEM lane
    const int wq = warp & 3;
    const float wv = P.norm_w ? bf2f(P.norm_w[u]) : 1.f;
    float* part = reinterpret_cast<float*>(smem + L::PART);
    // this thread's pieces of a chunk: row (u + 128 k) / 16, values 8 ((u + 128 k) % 16) .. + 7
    auto load_z = [&](int c, uint4 (&zz)[8]) {
      const int c0 = t_begin + c * GC, qn = min(GC, t_end - c0);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int idx = u + 128 * k, i = idx >> 4, cc = idx & 15;
        zz[k] = make_uint4(0u, 0u, 0u, 0u);
        if (P.z && i < qn)
          zz[k] = __ldg(reinterpret_cast<const uint4*>(P.z + static_cast<int64_t>(c0 + i) * P.z_t + j * P.z_h + cc * 8));
      }
    };
    uint4 zv[8], zn[8];
    if (nchunks > 0) load_z(0, zv);
    for (int c = 0; c < nchunks; ++c) {
      const int c0 = t_begin + c * GC;
      const int qn = min(GC, t_end - c0);
      float* ys = reinterpret_cast<float*>(smem + (c % L::NST) * L::STAGE + L::Q);  // [64][128] fp32, 32 KB
      if (c + 1 < nchunks) load_z(c + 1, zn);
      if (!and_bar(3, 128, wait_sleep(bar(WB_ODONE), c & 1, abort_flag, P.err))) break;
      tc_fence_after();
      float rsA = 1.f, rsB = 1.f;  // 1 / RMS of tokens lane and 32 + lane
      if (P.norm_w) {
        // per half of the chunk: squares over this warp's 32 rows, reduce-scattered so that lane l holds token l of the half
        float* pp = part + (c & 1) * 256;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t oh[32];
          tmem_ld32(t_lane + TM::O + 32 * h, oh);
          tmem_wait();
          float s[32];
#pragma unroll
          for (int k = 0; k < 32; ++k) s[k] = __uint_as_float(oh[k]) * __uint_as_float(oh[k]);
#pragma unroll
          for (int hs = 16; hs >= 1; hs >>= 1) {
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              if (k < hs) {
                const bool up = lane & hs;
                const float send = up ? s[k] : s[hs + k], keep = up ? s[hs + k] : s[k];
                s[k] = keep + __shfl_xor_sync(0xffffffffu, send, hs);
              }
            }
          }
          pp[wq * 64 + 32 * h + lane] = s[0];
        }
        asm volatile("bar.sync 3, 128;\n" ::: "memory");
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4) {
          t0 += pp[w4 * 64 + lane];
          t1 += pp[w4 * 64 + 32 + lane];
        }
        rsA = rsqrtf(t0 / static_cast<float>(GD) + P.eps);
        rsB = rsqrtf(t1 / static_cast<float>(GD) + P.eps);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t oh[32];
        tmem_ld32(t_lane + TM::O + 32 * h, oh);
        tmem_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float rs = __shfl_sync(0xffffffffu, h ? rsB : rsA, e);
          ys[(32 * h + e) * GD + u] = __uint_as_float(oh[e]) * rs * wv;
        }
      }
      tc_fence_before();
      arrive1(bar(WB_OFREE));  // O may be overwritten
      asm volatile("bar.sync 3, 128;\n" ::: "memory");
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int idx = u + 128 * k, i = idx >> 4, cc = idx & 15;
        if (i < qn) {
          const float4 a0 = *reinterpret_cast<const float4*>(ys + i * GD + cc * 8);
          const float4 a1 = *reinterpret_cast<const float4*>(ys + i * GD + cc * 8 + 4);
          float y[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          if (P.z) {
            const uint32_t zw[4] = {zv[k].x, zv[k].y, zv[k].z, zv[k].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 zf = unpack_bf16x2(zw[e]);
              y[2 * e] *= silu(zf.x);
              y[2 * e + 1] *= silu(zf.y);
            }
          }
          st16(P.out + static_cast<int64_t>(c0 + i) * P.o_t + j * P.o_h + cc * 8,
               make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                          pack_bf16x2(y[6], y[7])));
        }
      }
      asm volatile("bar.sync 3, 128;\n" ::: "memory");  // the staging is read: the stage may be reloaded
      if (u == 0) arrive1(bar(WB_EMPTY + c % L::NST));
#pragma unroll
      for (int k = 0; k < 8; ++k) zv[k] = zn[k];
    }
  }

  // teardown: every MMA has completed (bounded) before TMEM is released
  mbar_drain(bar(WB_DONE), 0);
  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem));
  }
}

// 3-D tensor map over [rows][mid][inner] bf16 (row stride s_t, middle stride s_mid, in elements), box 64 x 1 x 64
int gdn_map3(CUtensorMap* map, const void* base, int inner, int mid, int rows, int64_t s_mid, int64_t s_t) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(mid), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s_mid) * 2, static_cast<cuuint64_t>(s_t) * 2};
  cuuint32_t box[3] = {64, 1, 64};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill_tc: tensor map encode failed (%d)", (int)r);
  return MMP_OK;
}

template <typename Kern>
int smem_attr(Kern kern, int bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gdn_prefill_tc: smem attribute: %s", cudaGetErrorString(e));
    done[dev] = true;
  }
  return MMP_OK;
}

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" size_t mmp_gdn_prefill_workspace_size(int ntok, int nv) {
  if (ntok <= 0 || nv <= 0) return 0;
  return 2 * static_cast<size_t>(ntok) * nv * GC * sizeof(bf16);
}

extern "C" int mmp_gdn_prefill(const void* q, int64_t q_t, int64_t q_h, const void* k, int64_t k_t, int64_t k_h,
                               const void* v, int64_t v_t, int64_t v_h, const void* a, int64_t a_t,
                               const void* b, int64_t b_t, const float* A_log, const float* dt_bias,
                               const void* z, int64_t z_t, int64_t z_h, const void* norm_w, float eps,
                               float* state, int64_t s_line, int64_t s_head, int64_t s_row,
                               const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init,
                               void* out, int64_t o_t, int64_t o_h,
                               int nseq, int ntok, int nk, int nv, int dk, int dv, int lines, int* err, void* stream);

extern "C" int mmp_gdn_prefill_tc(const void* q, int64_t q_t, int64_t q_h, const void* k, int64_t k_t, int64_t k_h,
                                  const void* v, int64_t v_t, int64_t v_h, const void* a, int64_t a_t,
                                  const void* b, int64_t b_t, const float* A_log, const float* dt_bias,
                                  const void* z, int64_t z_t, int64_t z_h, const void* norm_w, float eps,
                                  float* state, int64_t s_line, int64_t s_head, int64_t s_row,
                                  const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init,
                                  void* out, int64_t o_t, int64_t o_h,
                                  int nseq, int ntok, int nk, int nv, int dk, int dv, int lines,
                                  void* workspace, size_t workspace_bytes, int* err, void* stream) {
  if (nseq == 0) return MMP_OK;
  if (!q || !k || !v || !a || !b || !state || !cu_seqlens || !state_idx || !out)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill_tc: null pointer");
  if (nseq < 0 || nseq > 65535 || ntok < 0 || nk <= 0 || nv <= 0 || nv % nk || nv > 65535 || lines <= 0)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill_tc: bad sizes nseq=%d nk=%d nv=%d lines=%d", nseq, nk, nv, lines);
  if (dk != GD || dv != GD)
    return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_gdn_prefill_tc: head dims %d x %d (only 128 x 128)", dk, dv);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || q_t % 8 || q_h % 8 || k_t % 8 || k_h % 8 || v_t % 8 || v_h % 8)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill_tc: q, k and v rows must be 16-byte aligned");
  if (!aligned16(state) || s_line % 4 || s_head % 4 || s_row % 4)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill_tc: state rows must be 16-byte aligned");
  if (!aligned16(out) || o_t % 8 || o_h % 8 || (z && (!aligned16(z) || z_t % 8 || z_h % 8)))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill_tc: out and z rows must be 16-byte aligned");
  if (ntok == 0)  // every sequence is empty: only the state lines are written
    return mmp_gdn_prefill(q, q_t, q_h, k, k_t, k_h, v, v_t, v_h, a, a_t, b, b_t, A_log, dt_bias, z, z_t, z_h, norm_w,
                           eps, state, s_line, s_head, s_row, cu_seqlens, state_idx, has_init, out, o_t, o_h, nseq, ntok,
                           nk, nv, dk, dv, lines, err, stream);
  const size_t need = mmp_gdn_prefill_workspace_size(ntok, nv);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill_tc: a 16-byte aligned workspace of %zu bytes is needed", need);
  int rc = get_encoder();
  if (rc != MMP_OK) return rc;
  bf16* Tw = static_cast<bf16*>(workspace);
  bf16* Qmw = Tw + static_cast<size_t>(ntok) * nv * GC;
  CUtensorMap mq, mk, mv, mt, mqm;
  if ((rc = gdn_map3(&mq, q, GD, nk, ntok, q_h, q_t)) || (rc = gdn_map3(&mk, k, GD, nk, ntok, k_h, k_t)) ||
      (rc = gdn_map3(&mv, v, GD, nv, ntok, v_h, v_t)) ||
      (rc = gdn_map3(&mt, Tw, GC, nv, ntok, GC, static_cast<int64_t>(nv) * GC)) ||
      (rc = gdn_map3(&mqm, Qmw, GC, nv, ntok, GC, static_cast<int64_t>(nv) * GC)))
    return rc;
  GdnTcParams P{static_cast<const bf16*>(q), q_t, q_h, static_cast<const bf16*>(k), k_t, k_h,
                static_cast<const bf16*>(v), v_t, v_h, static_cast<const bf16*>(a), a_t,
                static_cast<const bf16*>(b), b_t, A_log, dt_bias,
                static_cast<const bf16*>(z), z_t, z_h, static_cast<const bf16*>(norm_w), eps,
                state, s_line, s_head, s_row, cu_seqlens, state_idx, has_init,
                static_cast<bf16*>(out), o_t, o_h, Tw, Qmw, nseq, ntok, nk, nv, lines, err};
  static bool attr_prep[64] = {}, attr_walk[64] = {};
  if ((rc = smem_attr(gdn_chunk_prep_kernel, PrepSmem::DYN, attr_prep)) ||
      (rc = smem_attr(gdn_walk_tc_kernel, WalkSmem::DYN, attr_walk)))
    return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int chunk_bound = (ntok + GC - 1) / GC + nseq - 1;  // at least the number of chunks over all sequences
  cudaError_t e = mmp::launch(gdn_chunk_prep_kernel, dim3(chunk_bound, nk), dim3(PTHR), PrepSmem::DYN, s, nullptr, 0,
                              mq, mk, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gdn_prefill_tc: chunk pass: %s", cudaGetErrorString(e));
  if ((rc = mmp_check_launch("mmp_gdn_prefill_tc (chunk pass)")) != MMP_OK) return rc;
  e = mmp::launch(gdn_walk_tc_kernel, dim3(nv, nseq), dim3(WTHR), WalkSmem::DYN, s, nullptr, 0, mq, mk, mv, mt, mqm, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gdn_prefill_tc: walk: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_gdn_prefill_tc (walk)");
}
