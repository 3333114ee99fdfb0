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
// chunks of 64 tokens in order; the fp32 state stays in shared memory. The four contractions per chunk
// (C B^T, masked . x, C S^T, x^T . B-weighted) are bf16 tensor-core MMAs (mma.m16n8k16, fp32 accumulate) fed by
// ldmatrix from 128-byte-swizzled shared memory. Initial state: the sequence's state line (or zeros);
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
  static constexpr int RB = N * 2;                    // bf16 row bytes of B / C / S_bf
  static constexpr int C_OFF = 0;                     // [QC][N] bf16
  static constexpr int B_OFF = C_OFF + QC * RB;       // [QC][N] bf16, later the weighted B
  static constexpr int X_OFF = B_OFF + QC * RB;       // [QC][PT] bf16 (row 128 bytes)
  static constexpr int M_OFF = X_OFF + QC * PT * 2;   // [QC][QC] bf16 (row 128 bytes)
  static constexpr int SB_OFF = M_OFF + QC * QC * 2;  // [PT][N] bf16 state copy
  static constexpr int S_OFF = SB_OFF + PT * RB;      // [PT][N] fp32 state
  static constexpr int CUM_OFF = S_OFF + PT * N * 4;  // [QC] fp32 cumulative log-decay
  static constexpr int DT_OFF = CUM_OFF + QC * 4;     // [QC] fp32 dt
  static constexpr int BYTES = DT_OFF + QC * 4;
};

template <typename ST, int N>
__global__ void __launch_bounds__(THR, 1) ssd_prefill_kernel(const SsdParams P) {
  using L = SsdSmem<N>;
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_trigger();
  pdl_wait();
  const int p0 = blockIdx.x * PT, h = blockIdx.y, seq = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int t_begin = P.cu_seqlens[seq], t_end = P.cu_seqlens[seq + 1];
  const int line = P.state_idx[seq];
  if (line < 0 || line >= P.lines) {
    if (tid == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const int grp = h / (P.nh / P.ngroups);
  const float A = P.A[h], Dh = P.D ? P.D[h] : 0.f, dtb = P.dt_bias ? P.dt_bias[h] : 0.f;
  float* sS = reinterpret_cast<float*>(smem + L::S_OFF);
  float* sCum = reinterpret_cast<float*>(smem + L::CUM_OFF);
  float* sDt = reinterpret_cast<float*>(smem + L::DT_OFF);
  const uint32_t base = sa(smem);
  ST* gstate = reinterpret_cast<ST*>(P.state) + line * P.s_line + h * P.s_head + static_cast<int64_t>(p0) * P.s_p;

  // initial state
  const bool init = P.has_init && P.has_init[seq];
  for (int i = tid; i < PT * N; i += THR) {
    const int r = i / N, n = i % N;
    const float v = (init && p0 + r < P.p) ? static_cast<float>(gstate[r * P.s_p + n]) : 0.f;
    sS[i] = v;  // and the bf16 copy that feeds the C S^T contraction
    *reinterpret_cast<bf16*>(smem + L::SB_OFF + swz(r, n >> 3, L::RB) + (n & 7) * 2) = f2bf(v);
  }

  for (int c0 = t_begin; c0 < t_end; c0 += QC) {
    const int qn = min(QC, t_end - c0);
    __syncthreads();  // previous chunk fully consumed
    // ---- loads: C, B rows (N bf16), x slice (PT bf16), dt
    constexpr int CPR = N / 8;  // 16-byte chunks per B/C row
    for (int i = tid; i < QC * CPR; i += THR) {
      const int r = i / CPR, c = i % CPR;
      const bool v = r < qn;
      const int64_t t = c0 + (v ? r : 0);
      cp16(base + L::C_OFF + swz(r, c, L::RB), P.C + t * P.C_t + grp * P.C_g + c * 8, v);
      cp16(base + L::B_OFF + swz(r, c, L::RB), P.B + t * P.B_t + grp * P.B_g + c * 8, v);
    }
    for (int i = tid; i < QC * (PT / 8); i += THR) {
      const int r = i / (PT / 8), c = i % (PT / 8);
      const bool v = r < qn && p0 + c * 8 < P.p;
      const int64_t t = c0 + (r < qn ? r : 0);
      cp16(base + L::X_OFF + swz(r, c, PT * 2), P.x + t * P.x_t + h * P.x_h + p0 + c * 8, v);
    }
    asm volatile("cp.async.commit_group;\n" ::);
    if (warp == 0) {
      // dt' = softplus(dt + bias) and the inclusive running sum of dt' A over the chunk (two tokens per lane)
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
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        sDt[lane * 2 + j] = d[j];
        sCum[lane * 2 + j] = excl + cs[j];
      }
    }
    asm volatile("cp.async.wait_group 0;\n" ::);
    __syncthreads();
    const float cum_last = sCum[qn - 1];

    // ---- G = C B^T (QC x QC), masked and weighted into M[t][s] = G exp(cum_t - cum_s) dt_s (s <= t)
    {
      const int r0 = (warp >> 1) * 16, s0 = (warp & 1) * 32;
      float acc[4][4] = {};
      const int mat = lane >> 3, r8 = lane & 7;
#pragma unroll 4
      for (int k = 0; k < N / 16; ++k) {
        uint32_t a[4], b[2][4];
        ldsm_x4(base + L::C_OFF + swz(r0 + (mat & 1) * 8 + r8, k * 2 + (mat >> 1), L::RB), a);
#pragma unroll
        for (int np = 0; np < 2; ++np)
          ldsm_x4(base + L::B_OFF + swz(s0 + np * 16 + (mat >> 1) * 8 + r8, k * 2 + (mat & 1), L::RB), b[np]);
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
    __syncthreads();

    // ---- y = M x + exp(cum_t) C S^T + D x for this chunk (QC tokens x PT rows)
    {
      const int r0 = (warp >> 1) * 16, c0p = (warp & 1) * 32;
      const int mat = lane >> 3, r8 = lane & 7;
      float yi[4][4] = {}, ys[4][4] = {};
#pragma unroll
      for (int k = 0; k < QC / 16; ++k) {  // intra-chunk: K = tokens s
        uint32_t a[4], b[2][4];
        ldsm_x4(base + L::M_OFF + swz(r0 + (mat & 1) * 8 + r8, k * 2 + (mat >> 1), QC * 2), a);
#pragma unroll
        for (int np = 0; np < 2; ++np)  // x is [s][pp]: transposed load gives the (k = s, n = pp) fragment
          ldsm_x4_t(base + L::X_OFF + swz(k * 16 + (mat & 1) * 8 + r8, (c0p + np * 16) / 8 + (mat >> 1), PT * 2), b[np]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma16816(yi[nt], a, b[nt >> 1][(nt & 1) * 2], b[nt >> 1][(nt & 1) * 2 + 1]);
      }
#pragma unroll 4
      for (int k = 0; k < N / 16; ++k) {  // state term: K = n
        uint32_t a[4], b[2][4];
        ldsm_x4(base + L::C_OFF + swz(r0 + (mat & 1) * 8 + r8, k * 2 + (mat >> 1), L::RB), a);
#pragma unroll
        for (int np = 0; np < 2; ++np)
          ldsm_x4(base + L::SB_OFF + swz(c0p + np * 16 + (mat >> 1) * 8 + r8, k * 2 + (mat & 1), L::RB), b[np]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma16816(ys[nt], a, b[nt >> 1][(nt & 1) * 2], b[nt >> 1][(nt & 1) * 2 + 1]);
      }
      const bf16* sX = reinterpret_cast<const bf16*>(smem + L::X_OFF);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int t = r0 + g + (e >> 1) * 8, pp = c0p + nt * 8 + 2 * tq;
          if (t >= qn || p0 + pp >= P.p) continue;
          const float dec = __expf(sCum[t]);
          const bf16* xr = reinterpret_cast<const bf16*>(smem + L::X_OFF + swz(t, pp >> 3, PT * 2)) + (pp & 7);
          (void)sX;
          const float y0 = yi[nt][e] + dec * ys[nt][e] + Dh * bf2f(xr[0]);
          const float y1 = yi[nt][e + 1] + dec * ys[nt][e + 1] + Dh * bf2f(xr[1]);
          *reinterpret_cast<uint32_t*>(P.out + static_cast<int64_t>(c0 + t) * P.o_t + h * P.o_h + p0 + pp) =
              pack_bf16x2(y0, y1);
        }
      }
    }
    __syncthreads();

    // ---- weight B rows in place: W[s][n] = B[s][n] exp(cum_last - cum_s) dt_s
    for (int i = tid; i < QC * CPR; i += THR) {
      const int r = i / CPR, c = i % CPR;
      const float w = r < qn ? __expf(cum_last - sCum[r]) * sDt[r] : 0.f;
      uint4* ptr = reinterpret_cast<uint4*>(smem + L::B_OFF + swz(r, c, L::RB));
      uint4 u = *ptr;
      float2 a0 = unpack_bf16x2(u.x), a1 = unpack_bf16x2(u.y), a2 = unpack_bf16x2(u.z), a3 = unpack_bf16x2(u.w);
      *ptr = make_uint4(pack_bf16x2(a0.x * w, a0.y * w), pack_bf16x2(a1.x * w, a1.y * w),
                        pack_bf16x2(a2.x * w, a2.y * w), pack_bf16x2(a3.x * w, a3.y * w));
    }
    __syncthreads();

    // ---- S = exp(cum_last) S + x^T W  (PT x N), K = tokens s
    {
      constexpr int NW = N / 2;            // columns per warp (2 warps across n)
      constexpr int NT = NW / 8;           // n-tiles per warp
      const int r0 = (warp & 3) * 16, n0 = (warp >> 2) * NW;
      const float dec = __expf(cum_last);
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int n = n0 + nt * 8 + 2 * tq;
        acc[nt][0] = dec * sS[(r0 + g) * N + n];
        acc[nt][1] = dec * sS[(r0 + g) * N + n + 1];
        acc[nt][2] = dec * sS[(r0 + g + 8) * N + n];
        acc[nt][3] = dec * sS[(r0 + g + 8) * N + n + 1];
      }
      const int mat = lane >> 3, r8 = lane & 7;
#pragma unroll
      for (int k = 0; k < QC / 16; ++k) {
        uint32_t a[4];
        // A[pp][s] from x[s][pp]: 8x8 blocks (pp 0-7, s 0-7), (pp 8-15, s 0-7), (pp 0-7, s 8-15), (pp 8-15, s 8-15)
        ldsm_x4_t(base + L::X_OFF + swz(k * 16 + (mat >> 1) * 8 + r8, r0 / 8 + (mat & 1), PT * 2), a);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
          uint32_t b[4];  // W[s][n]: transposed load gives (k = s, n) fragments for n-tiles 2np, 2np + 1
          ldsm_x4_t(base + L::B_OFF + swz(k * 16 + (mat & 1) * 8 + r8, (n0 + np * 16) / 8 + (mat >> 1), L::RB), b);
          mma16816(acc[2 * np], a, b[0], b[1]);
          mma16816(acc[2 * np + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int n = n0 + nt * 8 + 2 * tq;
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = r0 + g + (e >> 1) * 8;
          sS[r * N + n] = acc[nt][e];
          sS[r * N + n + 1] = acc[nt][e + 1];
          *reinterpret_cast<uint32_t*>(smem + L::SB_OFF + swz(r, n >> 3, L::RB) + (n & 7) * 2) =
              pack_bf16x2(acc[nt][e], acc[nt][e + 1]);
        }
      }
    }
  }
  __syncthreads();
  // final state -> the sequence's line
  for (int i = tid; i < PT * N; i += THR) {
    const int r = i / N, n = i % N;
    if (p0 + r < P.p) gstate[r * P.s_p + n] = static_cast<ST>(sS[i]);
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

extern "C" int mmp_ssd_prefill(const void* x, int64_t x_t, int64_t x_h, const void* dt, int64_t dt_t, int64_t dt_h,
                               const float* A, const float* D, const float* dt_bias,
                               const void* B, int64_t B_t, int64_t B_g, const void* C, int64_t C_t, int64_t C_g,
                               void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                               const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init,
                               void* out, int64_t o_t, int64_t o_h,
                               int nseq, int nh, int p, int N, int ngroups, int lines, int* err, void* stream) {
  if (nseq == 0) return MMP_OK;
  if (!x || !dt || !A || !B || !C || !state || !cu_seqlens || !state_idx || !out)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: null pointer");
  if (nseq < 0 || nseq > 65535 || nh <= 0 || nh > 65535 || p <= 0 || p % 8 || ngroups <= 0 || nh % ngroups || lines <= 0)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: bad sizes nh=%d p=%d ngroups=%d", nh, p, ngroups);
  if (!aligned16(x) || !aligned16(B) || !aligned16(C) || x_t % 8 || x_h % 8 || B_t % 8 || B_g % 8 || C_t % 8 || C_g % 8 ||
      (o_t | o_h) & 1 || (reinterpret_cast<uintptr_t>(out) & 3))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: x, B, C rows must be 16-byte aligned, out 4-byte aligned");
  if (state_dtype != MMP_F32 && state_dtype != MMP_BF16)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill: state dtype must be fp32 or bf16");
  SsdParams P{static_cast<const bf16*>(x), x_t, x_h, static_cast<const bf16*>(dt), dt_t, dt_h, A, D, dt_bias,
              static_cast<const bf16*>(B), B_t, B_g, static_cast<const bf16*>(C), C_t, C_g,
              state, s_line, s_head, s_p, cu_seqlens, state_idx, has_init,
              static_cast<bf16*>(out), o_t, o_h, nh, p, ngroups, lines, err};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool f32 = state_dtype == MMP_F32;
  switch (N) {
    case 64: return f32 ? launch_ssd<float, 64>(P, nseq, s) : launch_ssd<bf16, 64>(P, nseq, s);
    case 128: return f32 ? launch_ssd<float, 128>(P, nseq, s) : launch_ssd<bf16, 128>(P, nseq, s);
    case 256: return f32 ? launch_ssd<float, 256>(P, nseq, s) : launch_ssd<bf16, 256>(P, nseq, s);
  }
  return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_ssd_prefill: d_state %d not in {64, 128, 256}", N);
}
