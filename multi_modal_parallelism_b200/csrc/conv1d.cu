// Mamba-2 decode causal depthwise conv update (replaces vLLM causal_conv1d_update as called by
// harness/kernels.py:131-134 of the reference).
//
// One thread owns 8 consecutive channels of one sequence: 16-byte loads of x, of the W-1 state rows and of
// the bias, 8 * W taps of weights, 16-byte stores of the output and of the shifted state. Channel-strided
// state layouts (s_c != 1) take a scalar path.
#include "mmp_common.cuh"

namespace mmp {
namespace {

constexpr int MAX_W = 8;

struct ConvParams {
  const bf16* x; int64_t x_b;
  bf16* out; int64_t o_b;
  bf16* state; int64_t s_line, s_k, s_c;
  const bf16* w; const bf16* bias;
  const int32_t* idx; int pad_slot;
  int batch, rows, W, lines, silu;
  int* err;
};

template <int W>
__global__ void __launch_bounds__(128) conv_update_vec_kernel(const ConvParams P) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.y;
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= P.rows) return;
  const int line = P.idx ? P.idx[b] : b;
  bf16* op = P.out + b * P.o_b + c0;
  if (line == P.pad_slot) {
    st16(op, make_uint4(0, 0, 0, 0));
    return;
  }
  if (line < 0 || line >= P.lines) {
    flag_error(P.err, DEVERR_INDEX);
    return;
  }
  float win[W][8];
  bf16* sp = P.state + line * P.s_line + c0;
#pragma unroll
  for (int k = 0; k < W - 1; ++k) {
    uint4 u = ld16(sp + k * P.s_k);
    float2 a = unpack_bf16x2(u.x), bb = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
    win[k][0] = a.x; win[k][1] = a.y; win[k][2] = bb.x; win[k][3] = bb.y;
    win[k][4] = c.x; win[k][5] = c.y; win[k][6] = d.x; win[k][7] = d.y;
  }
  uint4 ux = ld16(P.x + b * P.x_b + c0);
  {
    float2 a = unpack_bf16x2(ux.x), bb = unpack_bf16x2(ux.y), c = unpack_bf16x2(ux.z), d = unpack_bf16x2(ux.w);
    win[W - 1][0] = a.x; win[W - 1][1] = a.y; win[W - 1][2] = bb.x; win[W - 1][3] = bb.y;
    win[W - 1][4] = c.x; win[W - 1][5] = c.y; win[W - 1][6] = d.x; win[W - 1][7] = d.y;
  }
  float acc[8];
  if (P.bias) {
    uint4 ub = ld16(P.bias + c0);
    float2 a = unpack_bf16x2(ub.x), bb = unpack_bf16x2(ub.y), c = unpack_bf16x2(ub.z), d = unpack_bf16x2(ub.w);
    acc[0] = a.x; acc[1] = a.y; acc[2] = bb.x; acc[3] = bb.y; acc[4] = c.x; acc[5] = c.y; acc[6] = d.x; acc[7] = d.y;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  }
  // weights [rows, W]: 8 channels x W taps are 8*W contiguous bf16
  const bf16* wp = P.w + c0 * W;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
#pragma unroll
    for (int k = 0; k < W; ++k) acc[j] = fmaf(bf2f(wp[j * W + k]), win[k][j], acc[j]);
  }
  if (P.silu) {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = silu(acc[j]);
  }
  // shift the state line (reads of this line are complete: only this thread touches these channels)
#pragma unroll
  for (int k = 0; k < W - 2; ++k) st16(sp + k * P.s_k, ld16(sp + (k + 1) * P.s_k));
  if (W >= 2) st16(sp + (W - 2) * P.s_k, ux);
  st16(op, make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                      pack_bf16x2(acc[6], acc[7])));
}

__global__ void __launch_bounds__(128) conv_update_scalar_kernel(const ConvParams P) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= P.rows) return;
  const int line = P.idx ? P.idx[b] : b;
  if (line == P.pad_slot) {
    P.out[b * P.o_b + c] = f2bf(0.f);
    return;
  }
  if (line < 0 || line >= P.lines) {
    flag_error(P.err, DEVERR_INDEX);
    return;
  }
  bf16* sp = P.state + line * P.s_line + c * P.s_c;
  const bf16 xin = P.x[b * P.x_b + c];
  float acc = P.bias ? bf2f(P.bias[c]) : 0.f;
  for (int k = 0; k < P.W - 1; ++k) acc = fmaf(bf2f(P.w[c * P.W + k]), bf2f(sp[k * P.s_k]), acc);
  acc = fmaf(bf2f(P.w[c * P.W + P.W - 1]), bf2f(xin), acc);
  if (P.silu) acc = silu(acc);
  for (int k = 0; k < P.W - 2; ++k) sp[k * P.s_k] = sp[(k + 1) * P.s_k];
  if (P.W >= 2) sp[(P.W - 2) * P.s_k] = xin;
  P.out[b * P.o_b + c] = f2bf(acc);
}

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" int mmp_conv1d_update(const void* x, int64_t x_b, void* out, int64_t o_b,
                                 void* state, int64_t s_line, int64_t s_k, int64_t s_c,
                                 const void* w, const void* bias, const int32_t* idx, int pad_slot,
                                 int batch, int rows, int W, int lines, int silu, int* err, void* stream) {
  if (batch == 0) return MMP_OK;
  if (!x || !out || !state || !w) return mmp_set_error(MMP_ERR_INVALID, "mmp_conv1d_update: null pointer");
  if (batch < 0 || batch > 65535 || rows <= 0 || W < 1 || W > MAX_W || lines <= 0)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_conv1d_update: bad sizes batch=%d rows=%d W=%d lines=%d", batch, rows, W, lines);
  ConvParams P{static_cast<const bf16*>(x), x_b, static_cast<bf16*>(out), o_b,
               static_cast<bf16*>(state), s_line, s_k, s_c,
               static_cast<const bf16*>(w), static_cast<const bf16*>(bias), idx, pad_slot,
               batch, rows, W, lines, silu, err};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = s_c == 1 && W == 4 && rows % 8 == 0 && aligned16(x) && aligned16(out) && aligned16(state) &&
                   (!bias || aligned16(bias)) && x_b % 8 == 0 && o_b % 8 == 0 && s_line % 8 == 0 && s_k % 8 == 0;
  if (vec) {
    dim3 grid((rows / 8 + 127) / 128, batch);
    cudaError_t e = mmp::launch(conv_update_vec_kernel<4>, grid, dim3(128), 0, s, nullptr, 0, P);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_conv1d_update: %s", cudaGetErrorString(e));
  } else {
    dim3 grid((rows + 127) / 128, batch);
    cudaError_t e = mmp::launch(conv_update_scalar_kernel, grid, dim3(128), 0, s, nullptr, 0, P);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_conv1d_update: %s", cudaGetErrorString(e));
  }
  return mmp_check_launch("mmp_conv1d_update");
}

// ---------------------------------------------------------------------------------------------------------
// Prefill: the causal depthwise conv over variable-length sequences (vLLM causal_conv1d_fn in the serving
// stack; the reference harness itself only decodes). Token t of a sequence starting at `start` sees inputs
// t-W+1 .. t; inputs before `start` come from the sequence's conv-state line (oldest first) when it has an
// initial state, else are zero. A second launch writes each sequence's last W-1 inputs back to its line.
namespace mmp {
namespace {

struct ConvPrefillParams {
  const bf16* x; int64_t x_t;
  bf16* out; int64_t o_t;
  bf16* state; int64_t s_line, s_k;  // channels contiguous
  const bf16* w; const bf16* bias;
  const int32_t* cu_seqlens; const int32_t* state_idx; const int32_t* has_init;
  int nseq, rows, lines, silu;
  int* err;
};

__device__ __forceinline__ int seq_of(const int32_t* cu, int nseq, int t) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void unpack8f(const uint4& u, float* f) {
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

constexpr int CONV_RUN = 32;  // tokens per thread
constexpr int CONV_PF = 8;    // token rows loaded ahead

// One thread: 8 channels over a run of CONV_RUN consecutive packed tokens (which may cross sequence ends). The
// last W-1 inputs live in registers, so each input row is read once; the weights (W taps x 8 channels, 64
// contiguous bytes) are read once per thread. A warp covers 256 contiguous channels of a token row.
template <int W>
__global__ void __launch_bounds__(128) conv_prefill_kernel(const ConvPrefillParams P, int ntok) {
  pdl_trigger();
  pdl_wait();
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= P.rows) return;
  const int t0 = blockIdx.y * CONV_RUN;
  const int t1 = min(t0 + CONV_RUN, ntok);
  float wk[W][8];
  {
    static_assert(W * 8 % 8 == 0, "taps x 8 channels in 16-byte loads");
    float wf[W * 8];
#pragma unroll
    for (int i = 0; i < W; ++i) unpack8f(ld16(P.w + static_cast<int64_t>(c0) * W + i * 8), wf + i * 8);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int k = 0; k < W; ++k) wk[k][j] = wf[j * W + k];  // w[c][k] for c = c0 + j
  }
  float bias[8];
  if (P.bias) {
    unpack8f(ld16(P.bias + c0), bias);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) bias[j] = 0.f;
  }
  int seq = seq_of(P.cu_seqlens, P.nseq, t0);
  int s_end = P.cu_seqlens[seq + 1];
  float win[W - 1][8];  // inputs t-W+1 .. t-1, oldest first
  // history of a sequence whose first token in this run is t: inputs before its start come from its
  // conv-state line (when it has an initial state) or are zero
  auto load_history = [&](int t) -> bool {
    const int start = P.cu_seqlens[seq];
    const int line = P.state_idx[seq];
    const bool init = P.has_init && P.has_init[seq];
    if (init && (line < 0 || line >= P.lines)) {
      flag_error(P.err, DEVERR_INDEX);
      return false;
    }
#pragma unroll
    for (int k = 0; k < W - 1; ++k) {
      const int u = t - (W - 1) + k;
      if (u >= start) {
        unpack8f(ld16(P.x + static_cast<int64_t>(u) * P.x_t + c0), win[k]);
      } else if (init) {
        unpack8f(ld16(P.state + line * P.s_line + (u - start + W - 1) * P.s_k + c0), win[k]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) win[k][j] = 0.f;
      }
    }
    return true;
  };
  if (!load_history(t0)) return;
  for (int tb = t0; tb < t1; tb += CONV_PF) {
    uint4 rows[CONV_PF];
#pragma unroll
    for (int i = 0; i < CONV_PF; ++i)
      if (tb + i < t1) rows[i] = ld16(P.x + static_cast<int64_t>(tb + i) * P.x_t + c0);
#pragma unroll
    for (int i = 0; i < CONV_PF; ++i) {
      const int t = tb + i;
      if (t >= t1) break;
      if (t >= s_end) {  // first token of a later sequence (skipping empty ones)
        while (seq < P.nseq - 1 && t >= P.cu_seqlens[seq + 1]) ++seq;
        s_end = P.cu_seqlens[seq + 1];
        if (t >= s_end) {  // offsets that do not cover the packed tokens
          flag_error(P.err, DEVERR_INDEX);
          return;
        }
        if (!load_history(t)) return;
      }
      float v[8], acc[8];
      unpack8f(rows[i], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float a = bias[j];
#pragma unroll
        for (int k = 0; k < W - 1; ++k) a = fmaf(wk[k][j], win[k][j], a);
        a = fmaf(wk[W - 1][j], v[j], a);
        acc[j] = P.silu ? silu(a) : a;
      }
#pragma unroll
      for (int k = 0; k < W - 2; ++k)
#pragma unroll
        for (int j = 0; j < 8; ++j) win[k][j] = win[k + 1][j];
#pragma unroll
      for (int j = 0; j < 8; ++j) win[W - 2][j] = v[j];
      st16(P.out + static_cast<int64_t>(t) * P.o_t + c0,
           make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                      pack_bf16x2(acc[6], acc[7])));
    }
  }
}

template <int W>
__global__ void __launch_bounds__(128) conv_prefill_state_kernel(const ConvPrefillParams P) {
  pdl_trigger();
  pdl_wait();
  const int seq = blockIdx.y;
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= P.rows) return;
  const int start = P.cu_seqlens[seq], end = P.cu_seqlens[seq + 1], len = end - start;
  const int line = P.state_idx[seq];
  if (line < 0 || line >= P.lines) {
    flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const bool init = P.has_init && P.has_init[seq];
  bf16* sp = P.state + line * P.s_line + c0;
  uint4 nv[W - 1];
#pragma unroll
  for (int j = 0; j < W - 1; ++j) {  // read everything first: short sequences shift the old line
    const int u = end - (W - 1) + j;
    if (u >= start) nv[j] = ld16(P.x + static_cast<int64_t>(u) * P.x_t + c0);
    else if (init) nv[j] = ld16(sp + (len + j) * P.s_k);
    else nv[j] = make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int j = 0; j < W - 1; ++j) st16(sp + j * P.s_k, nv[j]);
}

}  // namespace
}  // namespace mmp

extern "C" int mmp_conv1d_prefill(const void* x, int64_t x_t, void* out, int64_t o_t, void* state, int64_t s_line,
                                  int64_t s_k, const void* w, const void* bias, const int32_t* cu_seqlens,
                                  const int32_t* state_idx, const int32_t* has_init, int nseq, int ntok, int rows,
                                  int W, int lines, int silu, int* err, void* stream) {
  if (nseq == 0 || ntok == 0) return MMP_OK;
  if (!x || !out || !state || !w || !cu_seqlens || !state_idx)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_conv1d_prefill: null pointer");
  if (x == out) return mmp_set_error(MMP_ERR_INVALID, "mmp_conv1d_prefill: out must not alias x");
  if (nseq < 0 || nseq > 65535 || ntok < 0 || rows <= 0 || rows % 8 || W != 4 || lines <= 0 ||
      !aligned16(x) || !aligned16(out) || !aligned16(state) || (bias && !aligned16(bias)) || x_t % 8 || o_t % 8 ||
      s_line % 8 || s_k % 8 || !aligned16(w))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_conv1d_prefill: needs W == 4, rows %% 8 == 0, 16-byte aligned rows");
  ConvPrefillParams P{static_cast<const bf16*>(x), x_t, static_cast<bf16*>(out), o_t, static_cast<bf16*>(state), s_line,
                      s_k, static_cast<const bf16*>(w), static_cast<const bf16*>(bias), cu_seqlens, state_idx, has_init,
                      nseq, rows, lines, silu, err};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int bx = (rows / 8 + 127) / 128;
  const int runs = (ntok + mmp::CONV_RUN - 1) / mmp::CONV_RUN;
  if (bx > 65535 || runs > 65535) return mmp_set_error(MMP_ERR_INVALID, "mmp_conv1d_prefill: too many channels or tokens");
  cudaError_t e = mmp::launch(conv_prefill_kernel<4>, dim3(bx, runs), dim3(128), 0, s, nullptr, 0, P, ntok);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_conv1d_prefill: %s", cudaGetErrorString(e));
  e = mmp::launch(conv_prefill_state_kernel<4>, dim3(bx, nseq), dim3(128), 0, s, nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_conv1d_prefill(state): %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_conv1d_prefill");
}
