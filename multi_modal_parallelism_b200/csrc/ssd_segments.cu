// Mamba-2 prefill scan with balanced walks: each sequence's token range is cut at 64-token chunk boundaries into
// segments that the chunked scan (mmp_ssd_prefill) runs as independent sequences, so that the (head, segment)
// walks fill the SMs in fewer, fuller waves than one walk per (head, sequence); the segments are then joined.
//
// With cum_t the running sum of dt'_u A over segment k up to token t (dt' = softplus(dt + dt_bias)), the
// recurrence s_t = exp(dt'_t A) s_{t-1} + dt'_t x_t B_t^T, y_t = s_t C_t + D x_t gives, for a segment entered with
// state S_in and scanned from zero state into (y_local, S_local):
//   y_t = y_local_t + exp(cum_t) S_in C_t          S_out = exp(cum_last) S_in + S_local
// (Mamba-2's chunk-state passing, Dao & Gu 2024, applied to segments of chunks). Steps, all on the stream:
//   1. seg_init: the state line of a sequence that continues (has_init) is copied, as fp32, to the scratch line
//      of its first segment;
//   2. the chunked scan over the segments, states in the fp32 scratch lines (first segments from their copied
//      initial state, the others from zero);
//   3. seg_join, one CTA per (head, sequence): walks the sequence's later segments in order, adds
//      exp(cum_t) (C_t S_in^T) to their outputs (mma.m16n8k16 over 64-token chunks of C against the bf16 S_in)
//      and chains S_in forward in fp32; the final state goes to the sequence's state line.
// Which cuts to make is the host's choice (kernels.ssd_segment_plan); any cuts at chunk boundaries are exact up
// to rounding.
#include <algorithm>

#include "mmp_common.cuh"

namespace mmp {
namespace {

constexpr int JTHR = 256;  // 8 warps
constexpr int JQ = 64;     // tokens per correction chunk
constexpr int JP = 128;    // head dim the join handles (p)

struct SegParams {
  const bf16* dt; int64_t dt_t, dt_h;
  const float* A; const float* dt_bias;
  const bf16* C; int64_t C_t, C_g;
  float* scratch; int64_t sc_line, sc_head;  // [scratch lines][nh][p][N] fp32, a head's p x N contiguous
  void* state; int64_t s_line, s_head, s_p;  // the sequences' state lines
  const int32_t* vcu;                          // [nvirt + 1] token offsets of the segments
  const int32_t* seg0;                         // [nseq + 1]: sequence i owns segments [seg0[i], seg0[i + 1])
  const int32_t* state_idx; const int32_t* has_init;
  bf16* y; int64_t y_t, y_h;
  int nh, ngroups, N, lines, nvirt;
  int* err;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// a sequence that continues from its state line: that line, as fp32, into its first segment's scratch line
template <typename ST>
__global__ void __launch_bounds__(JTHR) seg_init_kernel(const SegParams P) {
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x, i = blockIdx.y;
  if (!P.has_init || !P.has_init[i]) return;
  const int line = P.state_idx[i], v0 = P.seg0[i];
  if (line < 0 || line >= P.lines || v0 < 0 || v0 >= P.nvirt) {
    if (threadIdx.x == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const ST* src = reinterpret_cast<const ST*>(P.state) + line * P.s_line + h * P.s_head;
  float* dst = P.scratch + v0 * P.sc_line + h * P.sc_head;
  for (int e = threadIdx.x; e < JP * P.N; e += JTHR) dst[e] = static_cast<float>(src[(e / P.N) * P.s_p + e % P.N]);
}

template <int N>
struct JoinSmem {
  static constexpr int RS = N * 2 + 16;          // padded row (bytes): ldmatrix rows land on distinct banks
  static constexpr int SB_OFF = 0;               // bf16 S_in [p rows][N]
  static constexpr int C_OFF = JP * RS;          // C chunk [64 tokens][N]
  static constexpr int CUM_OFF = C_OFF + JQ * RS;  // cum[64] fp32, carry
  static constexpr int BYTES = CUM_OFF + JQ * 4 + 16;
};

template <typename ST, int N>
__global__ void __launch_bounds__(JTHR, 2) seg_join_kernel(const SegParams P) {
  using L = JoinSmem<N>;
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x, i = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const int v0 = P.seg0[i], v1 = P.seg0[i + 1];
  const int line = P.state_idx[i];
  if (line < 0 || line >= P.lines || v0 < 0 || v1 > P.nvirt || v1 <= v0) {
    if (tid == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const int grp = h / (P.nh / P.ngroups);
  const float A = P.A[h], dtb = P.dt_bias ? P.dt_bias[h] : 0.f;
  float* S = P.scratch + v0 * P.sc_line + h * P.sc_head;  // the chained state, updated in place
  float* sCum = reinterpret_cast<float*>(smem + L::CUM_OFF);
  float* sCarry = sCum + JQ;
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  constexpr int EL = JP * N / (JTHR * 8);  // 8-element groups of S per thread

  for (int v = v0 + 1; v < v1; ++v) {
    // S_in (this thread's 8-element groups) as bf16 operand rows
    __syncthreads();  // the previous segment's MMAs are done with the operand
#pragma unroll 4
    for (int k = 0; k < EL; ++k) {
      const int e = (k * JTHR + tid) * 8, r = e / N, c = e % N;
      const float4 a = *reinterpret_cast<const float4*>(S + e), b = *reinterpret_cast<const float4*>(S + e + 4);
      *reinterpret_cast<uint4*>(smem + L::SB_OFF + r * L::RS + c * 2) =
          make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
    }
    if (tid == 0) *sCarry = 0.f;
    const int t_beg = P.vcu[v], t_end = P.vcu[v + 1];
    for (int c0 = t_beg; c0 < t_end; c0 += JQ) {
      const int qn = min(JQ, t_end - c0);
      __syncthreads();  // operand rows written / the previous chunk's MMAs and scan readers are done
      for (int ci = tid; ci < JQ * (N / 8); ci += JTHR) {
        const int t = ci / (N / 8), c = ci % (N / 8);
        uint4 val = make_uint4(0, 0, 0, 0);
        if (t < qn) val = ld16(P.C + static_cast<int64_t>(c0 + t) * P.C_t + grp * P.C_g + c * 8);
        *reinterpret_cast<uint4*>(smem + L::C_OFF + t * L::RS + c * 16) = val;
      }
      if (warp == 0) {  // inclusive running sum of dt' A over the segment, 2 tokens per lane
        float d[2], cs[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int r = lane * 2 + j;
          d[j] = r < qn ? softplus(bf2f(P.dt[static_cast<int64_t>(c0 + r) * P.dt_t + h * P.dt_h]) + dtb) * A : 0.f;
        }
        cs[0] = d[0];
        cs[1] = d[0] + d[1];
        float run = cs[1];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float u = __shfl_up_sync(0xffffffffu, run, o);
          if (lane >= o) run += u;
        }
        const float carry = *sCarry, excl = run - cs[1];
        sCum[lane * 2] = carry + excl + cs[0];
        sCum[lane * 2 + 1] = carry + excl + cs[1];
        const float total = __shfl_sync(0xffffffffu, run, 31);
        __syncwarp();
        if (lane == 0) *sCarry = carry + total;
      }
      __syncthreads();
      // [64 tokens x 128 p] = C [64 x N] S_in^T: warp w takes rows 16 (w & 3), columns 64 (w >> 2)
      const int mt = warp & 3, nb = warp >> 2;
      const int mat = lane >> 3, r8 = lane & 7;
      float acc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll 4
      for (int k = 0; k < N / 16; ++k) {
        uint32_t a[4];
        ldsm_x4(sbase + L::C_OFF + (mt * 16 + (mat & 1) * 8 + r8) * L::RS + (k * 2 + (mat >> 1)) * 16, a);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b[4];
          ldsm_x4(sbase + L::SB_OFF + (nb * 64 + np * 16 + (mat >> 1) * 8 + r8) * L::RS + (k * 2 + (mat & 1)) * 16, b);
          mma16816(acc[2 * np], a, b[0], b[1]);
          mma16816(acc[2 * np + 1], a, b[2], b[3]);
        }
      }
      const int t0 = mt * 16 + g, t1 = t0 + 8;
      const float e0 = __expf(sCum[t0]), e1 = __expf(sCum[t1]);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int pc = nb * 64 + n * 8 + 2 * tq;
        if (t0 < qn) {
          uint32_t* yp = reinterpret_cast<uint32_t*>(P.y + static_cast<int64_t>(c0 + t0) * P.y_t + h * P.y_h + pc);
          const float2 o = unpack_bf16x2(*yp);
          *yp = pack_bf16x2(fmaf(e0, acc[n][0], o.x), fmaf(e0, acc[n][1], o.y));
        }
        if (t1 < qn) {
          uint32_t* yp = reinterpret_cast<uint32_t*>(P.y + static_cast<int64_t>(c0 + t1) * P.y_t + h * P.y_h + pc);
          const float2 o = unpack_bf16x2(*yp);
          *yp = pack_bf16x2(fmaf(e1, acc[n][2], o.x), fmaf(e1, acc[n][3], o.y));
        }
      }
    }
    // chain: S_out = exp(cum over the segment) S_in + S_local (this thread's groups only: no cross-thread reads)
    __syncthreads();  // the segment's carry is final
    const float dec = __expf(*sCarry);
    const float* Sl = P.scratch + v * P.sc_line + h * P.sc_head;
#pragma unroll 4
    for (int k = 0; k < EL; ++k) {
      const int e = (k * JTHR + tid) * 8;
#pragma unroll
      for (int q = 0; q < 8; q += 4) {
        float4 a = *reinterpret_cast<const float4*>(S + e + q);
        const float4 b = *reinterpret_cast<const float4*>(Sl + e + q);
        a = make_float4(fmaf(dec, a.x, b.x), fmaf(dec, a.y, b.y), fmaf(dec, a.z, b.z), fmaf(dec, a.w, b.w));
        *reinterpret_cast<float4*>(S + e + q) = a;
      }
    }
  }
  // the sequence's final state to its line
  ST* dst = reinterpret_cast<ST*>(P.state) + line * P.s_line + h * P.s_head;
#pragma unroll 4
  for (int k = 0; k < EL; ++k) {
    const int e = (k * JTHR + tid) * 8, r = e / N, c = e % N;
#pragma unroll
    for (int q = 0; q < 8; ++q) dst[r * P.s_p + c + q] = static_cast<ST>(S[e + q]);
  }
}

template <typename ST, int N>
int launch_join(const SegParams& P, int nseq, cudaStream_t s) {
  using L = JoinSmem<N>;
  auto kern = seg_join_kernel<ST, N>;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssd_prefill_seg: smem attribute: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  cudaError_t e = mmp::launch(kern, dim3(P.nh, nseq), dim3(JTHR), L::BYTES, s, nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssd_prefill_seg: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_ssd_prefill_seg (join)");
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
                               int nseq, int ntok, int nh, int p, int N, int ngroups, int lines, int* err,
                               void* stream);

extern "C" int mmp_ssd_prefill_seg(const void* x, int64_t x_t, int64_t x_h, const void* dt, int64_t dt_t,
                                   int64_t dt_h, const float* A, const float* D, const float* dt_bias,
                                   const void* B, int64_t B_t, int64_t B_g, const void* C, int64_t C_t, int64_t C_g,
                                   void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                                   const int32_t* state_idx, const int32_t* has_init, void* out, int64_t o_t,
                                   int64_t o_h, const int32_t* vcu, const int32_t* vline, const int32_t* vinit,
                                   const int32_t* seg0, float* scratch, int scratch_lines, int nvirt, int nseq,
                                   int ntok, int nh, int p, int N, int ngroups, int lines, int* err, void* stream) {
  if (nseq == 0 || ntok == 0) return MMP_OK;
  if (!vcu || !vline || !vinit || !seg0 || !scratch || !state || !state_idx)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill_seg: null pointer");
  if (p != JP || (N != 64 && N != 128 && N != 256))
    return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_ssd_prefill_seg: head dim %d, d_state %d (128 and 64/128/256)", p, N);
  if (nseq < 0 || nvirt < nseq || nvirt > scratch_lines || nh <= 0 || ngroups <= 0 || nh % ngroups || lines <= 0 ||
      nh > 65535 || nseq > 65535 || nvirt > 65535 || s_p < N)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill_seg: bad sizes (nseq %d, segments %d, scratch lines %d)",
                         nseq, nvirt, scratch_lines);
  if (!x || !dt || !A || !B || !C || !out || !aligned16(x) || !aligned16(B) || !aligned16(C) || !aligned16(out) ||
      !aligned16(scratch) || x_t % 8 || x_h % 8 || B_t % 8 || B_g % 8 || C_t % 8 || C_g % 8 || o_t % 8 || o_h % 8)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill_seg: x, B, C, out and scratch rows must be 16-byte aligned");
  if (state_dtype != MMP_F32 && state_dtype != MMP_BF16)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssd_prefill_seg: state dtype must be fp32 or bf16");
  const int64_t sc_head = static_cast<int64_t>(p) * N, sc_line = sc_head * nh;
  SegParams P{static_cast<const bf16*>(dt), dt_t, dt_h, A, dt_bias, static_cast<const bf16*>(C), C_t, C_g,
              scratch, sc_line, sc_head, state, s_line, s_head, s_p, vcu, seg0, state_idx, has_init,
              static_cast<bf16*>(out), o_t, o_h, nh, ngroups, N, lines, nvirt, err};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool f32 = state_dtype == MMP_F32;
  // 1. initial states of continuing sequences into their first segments' scratch lines
  if (has_init) {
    cudaError_t e = f32 ? mmp::launch(seg_init_kernel<float>, dim3(nh, nseq), dim3(JTHR), 0, s, nullptr, 0, P)
                        : mmp::launch(seg_init_kernel<bf16>, dim3(nh, nseq), dim3(JTHR), 0, s, nullptr, 0, P);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssd_prefill_seg: %s", cudaGetErrorString(e));
    const int rc = mmp_check_launch("mmp_ssd_prefill_seg (init)");
    if (rc != MMP_OK) return rc;
  }
  // 2. the chunked scan over the segments, states in the fp32 scratch lines
  int rc = mmp_ssd_prefill(x, x_t, x_h, dt, dt_t, dt_h, A, D, dt_bias, B, B_t, B_g, C, C_t, C_g, scratch, MMP_F32,
                           sc_line, sc_head, N, vcu, vline, vinit, out, o_t, o_h, nvirt, ntok, nh, p, N, ngroups,
                           scratch_lines, err, stream);
  if (rc != MMP_OK) return rc;
  // 3. join: later segments' outputs corrected, states chained, final states to the sequences' lines
  switch (N) {
    case 64: return f32 ? launch_join<float, 64>(P, nseq, s) : launch_join<bf16, 64>(P, nseq, s);
    case 128: return f32 ? launch_join<float, 128>(P, nseq, s) : launch_join<bf16, 128>(P, nseq, s);
    default: return f32 ? launch_join<float, 256>(P, nseq, s) : launch_join<bf16, 256>(P, nseq, s);
  }
}
