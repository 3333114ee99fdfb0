// Mamba-2 decode selective-state update (replaces vLLM selective_state_update as called by
// harness/kernels.py:137-143 of the reference).
//
// HBM-bound: per (sequence, head) the p x N state tile is read and written once (fp32: 2 * p * N * 4 bytes).
// Layout of the work: CTA = (row block of one head of one sequence); each warp owns R "passes" of rows; a
// row of N values is covered by LPR lanes with 16-byte vectors, so a warp reads whole contiguous rows and
// every lane keeps R*VPL 16-byte loads in flight before it computes. B/C of the head's group and the
// per-head scalars (dt', exp(dt' A), D) are loaded once per CTA into registers; the y = s.C reduction is a
// butterfly over the LPR lanes of a row.
#include "mmp_common.cuh"

namespace mmp {
namespace {

struct SsuParams {
  void* state; int64_t s_line, s_head, s_p;
  const bf16* x; int64_t x_b, x_h;
  const bf16* dt; int64_t dt_b, dt_h;
  const float* A; const float* D; const float* dt_bias;
  const bf16* B; int64_t B_b, B_g;
  const bf16* C; int64_t C_b, C_g;
  const bf16* z; int64_t z_b, z_h;
  const int32_t* idx_in; const int32_t* idx_out; int pad_slot;
  bf16* out; int64_t o_b, o_h;
  int batch, nh, p, N, ngroups, lines, dt_softplus;
  int* err;
};

template <typename ST> struct Vec;
template <> struct Vec<float> {
  static constexpr int EV = 4;  // elements per 16-byte vector
  __device__ static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y); f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
  __device__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};
template <> struct Vec<bf16> {
  static constexpr int EV = 8;
  __device__ static void unpack(const uint4& u, float* f) {
    float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
  }
  __device__ static uint4 pack(const float* f) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
  }
};

// Load EV consecutive bf16 values starting at p (EV = 4: 8 bytes, EV = 8: 16 bytes) as floats.
template <int EV>
__device__ __forceinline__ void load_bf16_vec(const bf16* p, float* f) {
  if constexpr (EV == 8) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    Vec<bf16>::unpack(u, f);
  } else {
    uint2 u = *reinterpret_cast<const uint2*>(p);
    float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  }
}

template <typename ST, int N, int WARPS>
struct SsuShape {
  static constexpr int EV = Vec<ST>::EV;
  static constexpr int VPL = (N >= EV * 32) ? N / (EV * 32) : 1;  // 16-byte vectors per lane per row
  static constexpr int LPR = N / (EV * VPL);                        // lanes per row
  static constexpr int RPP = 32 / LPR;                              // rows per warp pass
  static constexpr int R = (8 / VPL) > 0 ? 8 / VPL : 1;             // passes in flight per warp
  static constexpr int ROWS_WARP = R * RPP;
  static constexpr int ROWS_CTA = ROWS_WARP * WARPS;
  static_assert(LPR >= 1 && LPR <= 32 && 32 % LPR == 0, "row must map onto a power-of-two lane group");
};

template <typename ST, int N, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) ssu_decode_kernel(const SsuParams P) {
  pdl_trigger();
  using S = SsuShape<ST, N, WARPS>;
  constexpr int EV = S::EV, VPL = S::VPL, LPR = S::LPR, RPP = S::RPP, R = S::R;
  const int b = blockIdx.z, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, li = lane % LPR;
  const int row0 = blockIdx.x * S::ROWS_CTA + warp * S::ROWS_WARP + sub;

  // While the previous kernel finishes (the in-projection's epilogue, the conv), ask L2 for this CTA's state rows:
  // the state is the step's bulk traffic and no kernel before this one in a step writes it. Only a hint: the line
  // index read here feeds nothing but the prefetch address (lines outside [0, lines) are skipped), and every value
  // used below is read after the dependency wait.
  if (li == 0) {
    const int line = P.idx_in ? P.idx_in[b] : b;
    if (line >= 0 && line < P.lines && line != P.pad_slot) {
      const ST* rows = reinterpret_cast<const ST*>(P.state) + line * P.s_line + h * P.s_head;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = row0 + r * RPP;
        if (row < P.p) prefetch_l2_bulk(rows + row * P.s_p, N * sizeof(ST));
      }
    }
  }
  pdl_wait();

  const int line_in = P.idx_in ? P.idx_in[b] : b;
  bf16* outp = P.out + b * P.o_b + h * P.o_h;
  if (line_in == P.pad_slot) {
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r * RPP;
      if (li == 0 && row < P.p) outp[row] = f2bf(0.f);
    }
    return;
  }
  const int line_out = P.idx_out ? P.idx_out[b] : line_in;
  if (line_in < 0 || line_in >= P.lines || line_out < 0 || line_out >= P.lines) {
    if (threadIdx.x == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const int g = h / (P.nh / P.ngroups);

  const ST* src_state = reinterpret_cast<const ST*>(P.state) + line_in * P.s_line + h * P.s_head;
  ST* dst_state = reinterpret_cast<ST*>(P.state) + line_out * P.s_line + h * P.s_head;

  // Issue the state loads first: they are the only HBM traffic that matters.
  uint4 raw[R][VPL];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r * RPP;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int n0 = (v * LPR + li) * EV;
      raw[r][v] = row < P.p ? ld_stream16(src_state + row * P.s_p + n0) : make_uint4(0, 0, 0, 0);
    }
  }

  // Per-head scalars and this lane's slice of B and C.
  float dtv = bf2f(P.dt[b * P.dt_b + h * P.dt_h]) + (P.dt_bias ? P.dt_bias[h] : 0.f);
  if (P.dt_softplus) dtv = softplus(dtv);
  const float dA = __expf(dtv * P.A[h]);
  const float Dh = P.D ? P.D[h] : 0.f;
  float Bv[VPL][EV], Cv[VPL][EV];
  const bf16* Bp = P.B + b * P.B_b + g * P.B_g;
  const bf16* Cp = P.C + b * P.C_b + g * P.C_g;
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const int n0 = (v * LPR + li) * EV;
    load_bf16_vec<EV>(Bp + n0, Bv[v]);
    load_bf16_vec<EV>(Cp + n0, Cv[v]);
  }
  const bf16* xp = P.x + b * P.x_b + h * P.x_h;
  float xv[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r * RPP;
    xv[r] = row < P.p ? bf2f(xp[row]) : 0.f;
  }

  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float dx = dtv * xv[r];
    float a = 0.f;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      float s[EV];
      Vec<ST>::unpack(raw[r][v], s);
#pragma unroll
      for (int e = 0; e < EV; ++e) {
        s[e] = fmaf(s[e], dA, dx * Bv[v][e]);
        a = fmaf(s[e], Cv[v][e], a);
      }
      raw[r][v] = Vec<ST>::pack(s);
    }
    acc[r] = a;
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r * RPP;
    if (row < P.p) {
#pragma unroll
      for (int v = 0; v < VPL; ++v) st_stream16(dst_state + row * P.s_p + (v * LPR + li) * EV, raw[r][v]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
  }
  if (li == 0) {
    const bf16* zp = P.z ? P.z + b * P.z_b + h * P.z_h : nullptr;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r * RPP;
      if (row < P.p) {
        float y = acc[r] + Dh * xv[r];
        if (zp) y *= silu(bf2f(zp[row]));
        outp[row] = f2bf(y);
      }
    }
  }
}

template <typename ST, int N>
int launch(const SsuParams& P, cudaStream_t stream) {
  constexpr int WARPS = 4;
  using S = SsuShape<ST, N, WARPS>;
  dim3 grid((P.p + S::ROWS_CTA - 1) / S::ROWS_CTA, P.nh, P.batch);
  cudaError_t e = mmp::launch(ssu_decode_kernel<ST, N, WARPS>, grid, dim3(WARPS * 32), 0, stream, nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_ssu_decode: launch failed: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_ssu_decode");
}

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" int mmp_ssu_decode(void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                              const void* x, int64_t x_b, int64_t x_h,
                              const void* dt, int64_t dt_b, int64_t dt_h,
                              const float* A, const float* D, const float* dt_bias,
                              const void* B, int64_t B_b, int64_t B_g,
                              const void* C, int64_t C_b, int64_t C_g,
                              const void* z, int64_t z_b, int64_t z_h,
                              const int32_t* idx_in, const int32_t* idx_out, int pad_slot,
                              void* out, int64_t o_b, int64_t o_h,
                              int batch, int nh, int p, int N, int ngroups, int lines, int dt_softplus,
                              int* err, void* stream) {
  if (batch == 0) return MMP_OK;
  if (!state || !x || !dt || !A || !B || !C || !out)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssu_decode: null pointer");
  if (batch < 0 || nh <= 0 || p <= 0 || ngroups <= 0 || nh % ngroups || lines <= 0 || batch > 65535 || nh > 65535)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssu_decode: bad sizes batch=%d nh=%d p=%d ngroups=%d lines=%d",
                         batch, nh, p, ngroups, lines);
  if (state_dtype != MMP_F32 && state_dtype != MMP_BF16)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssu_decode: state dtype must be fp32 or bf16");
  const int esz = state_dtype == MMP_F32 ? 4 : 2;
  const int ev = 16 / esz;
  if (!aligned16(state) || (s_line * esz) % 16 || (s_head * esz) % 16 || (s_p * esz) % 16 || N % ev)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssu_decode: state rows must be 16-byte aligned");
  const int bc_align = N >= 128 || state_dtype == MMP_BF16 ? 16 : 8;
  if ((reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(C)) % bc_align || (B_b * 2) % bc_align ||
      (B_g * 2) % bc_align || (C_b * 2) % bc_align || (C_g * 2) % bc_align)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_ssu_decode: B/C rows must be %d-byte aligned", bc_align);
  SsuParams P{state, s_line, s_head, s_p,
              static_cast<const bf16*>(x), x_b, x_h,
              static_cast<const bf16*>(dt), dt_b, dt_h,
              A, D, dt_bias,
              static_cast<const bf16*>(B), B_b, B_g,
              static_cast<const bf16*>(C), C_b, C_g,
              static_cast<const bf16*>(z), z_b, z_h,
              idx_in, idx_out, pad_slot,
              static_cast<bf16*>(out), o_b, o_h,
              batch, nh, p, N, ngroups, lines, dt_softplus, err};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (state_dtype == MMP_F32) {
    switch (N) {
      case 64: return launch<float, 64>(P, s);
      case 128: return launch<float, 128>(P, s);
      case 256: return launch<float, 256>(P, s);
    }
  } else {
    switch (N) {
      case 64: return launch<bf16, 64>(P, s);
      case 128: return launch<bf16, 128>(P, s);
      case 256: return launch<bf16, 256>(P, s);
    }
  }
  return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_ssu_decode: d_state %d not in {64, 128, 256}", N);
}
