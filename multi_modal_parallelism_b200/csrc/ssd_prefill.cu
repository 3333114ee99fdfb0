// Mamba-2 prefill: the chunked state-space-duality (SSD) scan over variable-length sequences (the prefill
// counterpart of selective_state_update; vLLM's mamba_chunk_scan_combined_varlen in the serving stack the
// reference measures, named in docs/stage1_elastic_mixer_parallelism_plan.md:160-161).
//
// For a sequence and head, with a_t = dt_t A (dt_t = softplus(dt + dt_bias)) and cum the running sum of a
// inside a chunk, a chunk of tokens t maps the incoming state S (p x N) to
//   y_t   = sum_{s<=t} (C_t . B_s) exp(cum_t - cum_s) dt_s x_s  +  exp(cum_t) C_t S^T  +  D x_t
//   S_out = exp(cum_last) S + sum_s x_s (outer) B_s exp(cum_last - cum_s) dt_s
// which is the recurrence s_t = exp(a_t) s_{t-1} + dt_t x_t B_t^T, y_t = s_t C_t + D x_t unrolled over the
// chunk (Dao & Gu 2024). One CTA owns a 64-row slice of one head's p dimension for one sequence and walks its
// chunks of 64 tokens in order; the fp32 state lives in the warps' mma accumulators for the whole walk, and
// the next chunk's C, B and x are loaded (cp.async, two stages) under the current chunk's math. The four
// contractions per chunk (C B^T, x^T . M^T, S . C^T, x^T . B-weighted) are bf16 tensor-core MMAs
// (mma.m16n8k16, fp32 accumulate) fed by ldmatrix from 128-byte-swizzled shared memory. Initial state: the sequence's state line (or zeros);
// final state: written back to it.
#include <algorithm>

#include "mmp_common.cuh"

namespace mmp {
namespace {

constexpr int QC = 64;    // tokens per chunk
constexpr int PT = 64;    // p rows per CTA
constexpr int THR = 256;  // 8 warps

struct SsdParams {
  const bf16* x; int64_t x_t, x_h;      // [T, nh, p]
  const bf16* dt; int64_t dt_t, dt_h;   // [T, nh] raw (before bias / softplus)
  const float* A; const float* D; const float* dt_bias;
  const bf16* B; int64_t B_t, B_g;      // [T, G, N]
  const bf16* C; int64_t C_t, C_g;
  void* state; int64_t s_line, s_head, s_p;
  const int32_t* cu_seqlens;            // [nseq + 1]
  const int32_t* state_idx;             // [nseq]
  const int32_t* has_init;              // [nseq] or null (= no initial state)
  bf16* out; int64_t o_t, o_h;
  int nh, p, ngroups, lines;
  int* err;
};

__device__ __forceinline__ uint32_t sa(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// 16-byte chunk c of row r in a row of `row_bytes` (multiple of 128), XOR-swizzled inside each 128-byte group
__device__ __forceinline__ uint32_t swz(int r, int c, int row_bytes) { return r * row_bytes + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}

template <int N>
struct SsdSmem {
  static constexpr int RB = N * 2;                    // bf16 row bytes of B / C
  static constexpr int CB_BYTES = QC * RB;            // one chunk of C or B
  static constexpr int X_BYTES = QC * PT * 2;         // one chunk of x (row 128 bytes)
  static constexpr int STAGE = 2 * CB_BYTES + X_BYTES;  // C | B | x of one chunk; two stages
  static constexpr int M_OFF = 2 * STAGE;             // [QC][QC] bf16 masked, weighted C B^T
  static constexpr int YLD = QC + 8;                  // fp32 row stride of the partial exchange
  static constexpr int YP_OFF = M_OFF + QC * QC * 2;  // [PT][YLD] fp32 partials; then the y tile [QC][PT+8] bf16
  static constexpr int YT_LD = (PT + 8) * 2;          // byte row stride of the y tile
  static constexpr int CUM_OFF = YP_OFF + PT * YLD * 4;  // [QC] fp32 cumulative log-decay
  static constexpr int DT_OFF = CUM_OFF + QC * 4;     // [QC] fp32 dt
  static constexpr int BYTES = DT_OFF + QC * 4;
  static_assert(QC * YT_LD <= PT * YLD * 4, "y tile fits the partial buffer");
};

// Warp roles (8 warps): warp w owns state rows p = (w & 3) * 16 .. +15 and state columns n in half (w >> 2),
// as mma accumulators in registers for the whole walk. Its output work is the y^T tile of the same 16 rows
// and token half (w >> 2): the state term sum_n S[p][n] C[t][n] is computed over its own column half for all
// 64 tokens (A operand = the accumulators repacked to bf16), and the two warps of a row tile swap the halves
// they do not own through shared memory.
template <typename ST, int N>
__global__ void __launch_bounds__(THR, 1) ssd_prefill_kernel(const SsdParams P) {
  using L = SsdSmem<N>;
  constexpr int NH = N / 2;   // state columns per warp
  constexpr int NT = NH / 8;  // state n8-tiles per warp
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_trigger();
  pdl_wait();
  const int p0 = blockIdx.x * PT, h = blockIdx.y, seq = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3, mat = lane >> 3, r8 = lane & 7;
  const int t_begin = P.cu_seqlens[seq], t_end = P.cu_seqlens[seq + 1];
  const int line = P.state_idx[seq];
  if (line < 0 || line >= P.lines) {
    if (tid == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const int grp = h / (P.nh / P.ngroups);
  const float A = P.A[h], Dh = P.D ? P.D[h] : 0.f, dtb = P.dt_bias ? P.dt_bias[h] : 0.f;
  float* sCum = reinterpret_cast<float*>(smem + L::CUM_OFF);
  float* sDt = reinterpret_cast<float*>(smem + L::DT_OFF);
  float* sYP = reinterpret_cast<float*>(smem + L::YP_OFF);
  const uint32_t base = sa(smem);
  ST* gstate = reinterpret_cast<ST*>(P.state) + line * P.s_line + h * P.s_head + static_cast<int64_t>(p0) * P.s_p;
  const int pr = (warp & 3) * 16;      // state / output rows of this warp
  const int half = warp >> 2;
  const int nh0 = half * NH;           // state columns of this warp
  const int th0 = half * (QC / 2);     // output tokens of this warp

  // ---- initial state into the accumulators (rows pr+g, pr+g+8; columns nh0 + nt*8 + 2tq, +1)
  float S[NT][4];
  {
    const bool init = P.has_init && P.has_init[seq];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nh0 + nt * 8 + 2 * tq;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = pr + g + (e >> 1) * 8;
        S[nt][e] = (init && p0 + r < P.p) ? static_cast<float>(gstate[r * P.s_p + n + (e & 1)]) : 0.f;
      }
    }
  }

  constexpr int CPR = N / 8;  // 16-byte chunks per B/C row
  auto issue = [&](int c0, int stage) {
    const int qn = min(QC, t_end - c0);
    const uint32_t sC = base + stage * L::STAGE, sB = sC + L::CB_BYTES, sX = sB + L::CB_BYTES;
    for (int i = tid; i < QC * CPR; i += THR) {
      const int r = i / CPR, c = i % CPR;
      const bool v = r < qn;
      const int64_t t = c0 + (v ? r : 0);
      cp16(sC + swz(r, c, L::RB), P.C + t * P.C_t + grp * P.C_g + c * 8, v);
      cp16(sB + swz(r, c, L::RB), P.B + t * P.B_t + grp * P.B_g + c * 8, v);
    }
    for (int i = tid; i < QC * (PT / 8); i += THR) {
      const int r = i / (PT / 8), c = i % (PT / 8);
      const bool v = r < qn && p0 + c * 8 < P.p;
      const int64_t t = c0 + (r < qn ? r : 0);
      cp16(sX + swz(r, c, PT * 2), P.x + t * P.x_t + h * P.x_h + p0 + c * 8, v);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };
  float dnext[2] = {0.f, 0.f};  // warp 0: raw dt of tokens 2 lane, 2 lane + 1 of the next chunk
  auto load_dt = [&](int c0) {
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = lane * 2 + j;
        dnext[j] = c0 + r < t_end ? bf2f(P.dt[static_cast<int64_t>(c0 + r) * P.dt_t + h * P.dt_h]) : 0.f;
      }
    }
  };
  if (t_begin < t_end) {
    issue(t_begin, 0);
    load_dt(t_begin);
  }

  int stage = 0;
  for (int c0 = t_begin; c0 < t_end; c0 += QC, stage ^= 1) {
    const int qn = min(QC, t_end - c0);
    if (warp == 0) {
      // dt' = softplus(dt + bias) and the inclusive running sum of dt' A over the chunk (two tokens per lane)
      float d[2], cs[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) d[j] = lane * 2 + j < qn ? softplus(dnext[j] + dtb) : 0.f;
      cs[0] = d[0] * A;
      cs[1] = cs[0] + d[1] * A;
      float run = cs[1];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, run, o);
        if (lane >= o) run += v;
      }
      const float excl = run - cs[1];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        sDt[lane * 2 + j] = d[j];
        sCum[lane * 2 + j] = excl + cs[j];
      }
    }
    // next chunk's loads run under this chunk's math (its stage was released by the last barrier)
    if (c0 + QC < t_end) {
      issue(c0 + QC, stage ^ 1);
      load_dt(c0 + QC);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();
    const float cum_last = sCum[qn - 1];
    const uint32_t sC = base + stage * L::STAGE, sB = sC + L::CB_BYTES, sX = sB + L::CB_BYTES;
    uint8_t* pB = smem + stage * L::STAGE + L::CB_BYTES;

    // ---- G = C B^T (QC x QC), masked and weighted into M[t][s] = G exp(cum_t - cum_s) dt_s (s <= t)
    {
      const int r0 = (warp >> 1) * 16, s0 = (warp & 1) * 32;
      float acc[4][4] = {};
#pragma unroll 4
      for (int k = 0; k < N / 16; ++k) {
        uint32_t a[4], b[2][4];
        ldsm_x4(sC + swz(r0 + (mat & 1) * 8 + r8, k * 2 + (mat >> 1), L::RB), a);
#pragma unroll
        for (int np = 0; np < 2; ++np)
          ldsm_x4(sB + swz(s0 + np * 16 + (mat >> 1) * 8 + r8, k * 2 + (mat & 1), L::RB), b[np]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma16816(acc[nt], a, b[nt >> 1][(nt & 1) * 2], b[nt >> 1][(nt & 1) * 2 + 1]);
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int t = r0 + g + (e >> 1) * 8, s = s0 + nt * 8 + 2 * tq;
          float v0 = 0.f, v1 = 0.f;
          if (s <= t) v0 = acc[nt][e] * __expf(sCum[t] - sCum[s]) * sDt[s];
          if (s + 1 <= t) v1 = acc[nt][e + 1] * __expf(sCum[t] - sCum[s + 1]) * sDt[s + 1];
          *reinterpret_cast<uint32_t*>(smem + L::M_OFF + swz(t, s >> 3, QC * 2) + (s & 7) * 2) = pack_bf16x2(v0, v1);
        }
      }
    }

    // ---- state term, this warp's column half, all tokens: ys[p][t] = sum_{n in half} S[p][n] C[t][n]
    float ys[QC / 8][4] = {};
#pragma unroll
    for (int kk = 0; kk < NH / 16; ++kk) {
      uint32_t a[4];  // accumulator n8-tiles 2kk, 2kk+1 are the A fragment of this k16 step
      a[0] = pack_bf16x2(S[2 * kk][0], S[2 * kk][1]);
      a[1] = pack_bf16x2(S[2 * kk][2], S[2 * kk][3]);
      a[2] = pack_bf16x2(S[2 * kk + 1][0], S[2 * kk + 1][1]);
      a[3] = pack_bf16x2(S[2 * kk + 1][2], S[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < QC / 16; ++np) {
        uint32_t b[4];  // C[t][n]: rows t, k = n
        ldsm_x4(sC + swz(np * 16 + (mat >> 1) * 8 + r8, (nh0 + kk * 16) / 8 + (mat & 1), L::RB), b);
        mma16816(ys[2 * np], a, b[0], b[1]);
        mma16816(ys[2 * np + 1], a, b[2], b[3]);
      }
    }
    // hand the other token half to the partner warp
#pragma unroll
    for (int nt = 0; nt < QC / 8; ++nt) {
      if ((nt >= QC / 16) == (half == 1)) continue;  // own half
      const int t = nt * 8 + 2 * tq;
#pragma unroll
      for (int e = 0; e < 4; e += 2)
        *reinterpret_cast<float2*>(sYP + (pr + g + (e >> 1) * 8) * L::YLD + t) = make_float2(ys[nt][e], ys[nt][e + 1]);
    }
    __syncthreads();

    // ---- intra-chunk term for this warp's token half: yi[p][t] = sum_s x[s][p] M[t][s]; combine
    float yv[QC / 16][4];
    {
      float yi[QC / 16][4] = {};
#pragma unroll
      for (int ks = 0; ks < QC / 16; ++ks) {
        uint32_t a[4];  // A[p][s] from x[s][p]: transposed 8x8 blocks
        ldsm_x4_t(sX + swz(ks * 16 + (mat >> 1) * 8 + r8, pr / 8 + (mat & 1), PT * 2), a);
#pragma unroll
        for (int np = 0; np < QC / 32; ++np) {
          uint32_t b[4];  // M[t][s]: rows t, k = s
          ldsm_x4(base + L::M_OFF + swz(th0 + np * 16 + (mat >> 1) * 8 + r8, ks * 2 + (mat & 1), QC * 2), b);
          mma16816(yi[2 * np], a, b[0], b[1]);
          mma16816(yi[2 * np + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < QC / 16; ++j) {
        float own[4];  // state-term partial of this warp's token half (static register indexing)
#pragma unroll
        for (int e = 0; e < 4; ++e) own[e] = half ? ys[QC / 16 + j][e] : ys[j][e];
        const int t = th0 + j * 8 + 2 * tq;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = pr + g + (e >> 1) * 8, tt = t + (e & 1);
          const float part = sYP[r * L::YLD + tt];
          const float xv = bf2f(*reinterpret_cast<const bf16*>(smem + stage * L::STAGE + 2 * L::CB_BYTES +
                                                                swz(tt, r >> 3, PT * 2) + (r & 7) * 2));
          yv[j][e] = yi[j][e] + __expf(sCum[tt]) * (own[e] + part) + Dh * xv;
        }
      }
    }
    // weight B rows in place for the state update: W[s][n] = B[s][n] exp(cum_last - cum_s) dt_s
    for (int i = tid; i < QC * CPR; i += THR) {
      const int r = i / CPR, c = i % CPR;
      const float w = r < qn ? __expf(cum_last - sCum[r]) * sDt[r] : 0.f;
      uint4* ptr = reinterpret_cast<uint4*>(pB + swz(r, c, L::RB));
      uint4 u = *ptr;
      float2 a0 = unpack_bf16x2(u.x), a1 = unpack_bf16x2(u.y), a2 = unpack_bf16x2(u.z), a3 = unpack_bf16x2(u.w);
      *ptr = make_uint4(pack_bf16x2(a0.x * w, a0.y * w), pack_bf16x2(a1.x * w, a1.y * w),
                        pack_bf16x2(a2.x * w, a2.y * w), pack_bf16x2(a3.x * w, a3.y * w));
    }
    __syncthreads();

    // ---- y tile [t][p] (bf16) into the partial buffer; S = exp(cum_last) S + x^T W
#pragma unroll
    for (int j = 0; j < QC / 16; ++j) {
      const int t = th0 + j * 8 + 2 * tq;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = pr + g + (e >> 1) * 8;
        *reinterpret_cast<bf16*>(smem + L::YP_OFF + (t + (e & 1)) * L::YT_LD + r * 2) = f2bf(yv[j][e]);
      }
    }
    {
      const float dec = __expf(cum_last);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[nt][e] *= dec;
#pragma unroll
      for (int k = 0; k < QC / 16; ++k) {
        uint32_t a[4];
        ldsm_x4_t(sX + swz(k * 16 + (mat >> 1) * 8 + r8, pr / 8 + (mat & 1), PT * 2), a);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
          uint32_t b[4];  // W[s][n]: transposed load gives (k = s, n) fragments for n-tiles 2np, 2np + 1
          ldsm_x4_t(sB + swz(k * 16 + (mat & 1) * 8 + r8, (nh0 + np * 16) / 8 + (mat >> 1), L::RB), b);
          mma16816(S[2 * np], a, b[0], b[1]);
          mma16816(S[2 * np + 1], a, b[2], b[3]);
        }
      }
    }
    __syncthreads();
    // ---- coalesced store of the y tile: 8 threads x 16 bytes per token row
    for (int i = tid; i < QC * (PT / 8); i += THR) {
      const int t = i / (PT / 8), c = i % (PT / 8);
      if (t < qn && p0 + c * 8 < P.p)
        st16(P.out + static_cast<int64_t>(c0 + t) * P.o_t + h * P.o_h + p0 + c * 8,
             *reinterpret_cast<const uint4*>(smem + L::YP_OFF + t * L::YT_LD + c * 16));
    }
  }
  // final state -> the sequence's line
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int n = nh0 + nt * 8 + 2 * tq;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = pr + g + (e >> 1) * 8;
      if (p0 + r < P.p) gstate[r * P.s_p + n + (e & 1)] = static_cast<ST>(S[nt][e]);
    }
  }
}

template <typename ST, int N>
int launch_ssd(const SsdParams& P, int nseq, cudaStream_t s) {
  using L = SsdSmem<N>;
  auto kern = ssd_prefill_kernel<ST, N>;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssd_prefill: smem attribute: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  dim3 grid((P.p + PT - 1) / PT, P.nh, nseq);
  cudaError_t e = mmp::launch(kern, grid, dim3(THR), L::BYTES, s, nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssd_prefill: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_ssd_prefill");
}

}  // namespace
}  // namespace mmp

using namespace mmp;

namespace mmp {
static int g_ssd_prefill_tc = 1;  // mmp_set_ssd_prefill_tc(0): the mma.sync kernel for every shape
int ssd_prefill_tc(const void* x, int64_t x_t, int64_t x_h, const void* dt, int64_t dt_t, int64_t dt_h, const float* A,
                   const float* D, const float* dt_bias, const void* B, int64_t B_t, int64_t B_g, const void* C,
                   int64_t C_t, int64_t C_g, void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                   const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init, void* out,
                   int64_t o_t, int64_t o_h, int nseq, int ntok, int nh, int p, int N, int ngroups, int lines, int* err,
                   cudaStream_t stream);
}  // namespace mmp

extern "C" int mmp_ssd_prefill(const void* x, int64_t x_t, int64_t x_h, const void* dt, int64_t dt_t, int64_t dt_h,
                               const float* A, const float* D, const float* dt_bias,
                               const void* B, int64_t B_t, int64_t B_g, const void* C, int64_t C_t, int64_t C_g,
                               void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                               const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init,
                               void* out, int64_t o_t, int64_t o_h,
                               int nseq, int ntok, int nh, int p, int N, int ngroups, int lines, int* err,
                               void* stream) {
  if (nseq == 0 || ntok == 0) return MMP_OK;
  if (!x || !dt || !A || !B || !C || !state || !cu_seqlens || !state_idx || !out)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: null pointer");
  if (nseq < 0 || nseq > 65535 || nh <= 0 || nh > 65535 || p <= 0 || p % 8 || ngroups <= 0 || nh % ngroups || lines <= 0)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: bad sizes nh=%d p=%d ngroups=%d", nh, p, ngroups);
  if (!aligned16(x) || !aligned16(B) || !aligned16(C) || x_t % 8 || x_h % 8 || B_t % 8 || B_g % 8 || C_t % 8 || C_g % 8 ||
      o_t % 8 || o_h % 8 || !aligned16(out))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: x, B, C and out rows must be 16-byte aligned");
  if (state_dtype != MMP_F32 && state_dtype != MMP_BF16)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: state dtype must be fp32 or bf16");
  SsdParams P{static_cast<const bf16*>(x), x_t, x_h, static_cast<const bf16*>(dt), dt_t, dt_h, A, D, dt_bias,
              static_cast<const bf16*>(B), B_t, B_g, static_cast<const bf16*>(C), C_t, C_g,
              state, s_line, s_head, s_p, cu_seqlens, state_idx, has_init,
              static_cast<bf16*>(out), o_t, o_h, nh, p, ngroups, lines, err};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ntok < 0) return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: ntok %d", ntok);
  // head dim 128 with d_state 128 / 256, head dim 64 with d_state 128: the tcgen05 kernel (ssd_prefill_tc.cu)
  const int tc = !g_ssd_prefill_tc ? MMP_ERR_UNSUPPORTED : ssd_prefill_tc(x, x_t, x_h, dt, dt_t, dt_h, A, D, dt_bias, B, B_t, B_g, C, C_t, C_g, state,
                                state_dtype, s_line, s_head, s_p, cu_seqlens, state_idx, has_init, out, o_t, o_h,
                                                         nseq, ntok, nh, p, N, ngroups, lines, err, s);
  if (tc != MMP_ERR_UNSUPPORTED) return tc;
  const bool f32 = state_dtype == MMP_F32;
  switch (N) {
    case 64: return f32 ? launch_ssd<float, 64>(P, nseq, s) : launch_ssd<bf16, 64>(P, nseq, s);
    case 128: return f32 ? launch_ssd<float, 128>(P, nseq, s) : launch_ssd<bf16, 128>(P, nseq, s);
    case 256: return f32 ? launch_ssd<float, 256>(P, nseq, s) : launch_ssd<bf16, 256>(P, nseq, s);
  }
  return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_ssd_prefill: d_state %d not in {64, 128, 256}", N);
}

extern "C" int mmp_set_ssd_prefill_tc(int enable) {
  const int prev = mmp::g_ssd_prefill_tc;
  mmp::g_ssd_prefill_tc = enable ? 1 : 0;
  return prev;
}
