// RMSNorm (+ fused residual add) and the Mamba-2 gated RMSNorm (replace vLLM rms_norm and
// rms_norm_gated / the tensor-parallel torch path, harness/kernels.py:26-28,40-52 of the reference).
//
// One CTA per row (per row and group for the gated norm); 16-byte vectors of 8 bf16; fp32 statistics. The
// row is read twice (statistics, then normalise): the second read hits L1/L2, so HBM traffic stays one
// read of the inputs plus one write.
#include "mmp_common.cuh"

namespace mmp {
namespace {

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
}

struct RmsParams {
  const bf16* x; int64_t x_b;
  const bf16* res; int64_t r_b;
  bf16* sum_out; int64_t s_b;
  const bf16* w;
  bf16* out; int64_t o_b;
  int hidden;
  float eps;
};

// Up to MAXV vectors per thread are kept in registers between the two passes.
template <int MAXV>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const RmsParams P) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nvec = P.hidden / 8;
  float v[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      unpack8(ld16(P.x + row * P.x_b + vi * 8), v[i]);
      if (P.res) {
        float r[8];
        unpack8(ld16(P.res + row * P.r_b + vi * 8), r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[j];
        // the stored sum is bf16; normalise the stored value so sum_out and out agree
        uint4 packed = pack8(v[i]);
        if (P.sum_out) st16(P.sum_out + row * P.s_b + vi * 8, packed);
        unpack8(packed, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[i][j], v[i][j], ss);
    }
  }
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(total / P.hidden + P.eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      float w[8], o[8];
      unpack8(ld16(P.w + vi * 8), w);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv * w[j];
      st16(P.out + row * P.o_b + vi * 8, pack8(o));
    }
  }
}

struct GnParams {
  const bf16* y; int64_t y_b;
  const bf16* z; int64_t z_b;
  const bf16* w;
  bf16* out; int64_t o_b;
  float* sumsq;
  int D, group_size, mode;
  float count, eps;
};

// grid: (groups, rows). mode 0 = local, 1 = write partial sums, 2 = apply given sums, 3 = write partial sums and
// the gated, weighted values unnormalised (the caller scales the rows once the sums are complete).
template <int MAXV>
__global__ void __launch_bounds__(256) gated_rmsnorm_kernel(const GnParams P) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int grp = blockIdx.x, row = blockIdx.y, ngroups = gridDim.x;
  const int nvec = P.group_size / 8;
  const int base = grp * P.group_size;
  float g[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      float yv[8], zv[8];
      unpack8(ld16(P.y + row * P.y_b + base + vi * 8), yv);
      unpack8(ld16(P.z + row * P.z_b + base + vi * 8), zv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        g[i][j] = yv[j] * silu(zv[j]);
        ss = fmaf(g[i][j], g[i][j], ss);
      }
    }
  }
  float total;
  if (P.mode == 2) {
    total = P.sumsq[row * ngroups + grp];
  } else {
    total = block_sum(ss, red);
    if (P.mode == 1 || P.mode == 3) {
      if (threadIdx.x == 0) P.sumsq[row * ngroups + grp] = total;
      if (P.mode == 1) return;
    }
  }
  const float cnt = P.mode == 2 ? P.count : static_cast<float>(P.group_size);
  const float inv = P.mode == 3 ? 1.f : rsqrtf(total / cnt + P.eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      float w[8], o[8];
      unpack8(ld16(P.w + base + vi * 8), w);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = g[i][j] * inv * w[j];
      st16(P.out + row * P.o_b + base + vi * 8, pack8(o));
    }
  }
}

// x[r, :] *= rsqrt(sumsq[r] / count + eps), in place (bf16 rows, fp32 sums): the deferred normalisation of a
// partial product computed from unnormalised gated values. grid: rows; 16-byte vectors.
__global__ void __launch_bounds__(256) scale_rows_kernel(bf16* x, int64_t ld, const float* sumsq, int cols,
                                                         float count, float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const float s = rsqrtf(sumsq[row] / count + eps);
  bf16* xr = x + row * ld;
  for (int v = threadIdx.x; v < cols / 8; v += blockDim.x) {
    float f[8];
    unpack8(ld16(xr + v * 8), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] *= s;
    st16(xr + v * 8, pack8(f));
  }
}

bool rows_ok(const void* p, int64_t stride) { return p == nullptr || (aligned16(p) && stride % 8 == 0); }

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" int mmp_rmsnorm(const void* x, int64_t x_b, const void* residual, int64_t r_b, void* sum_out, int64_t s_b,
                           const void* w, void* out, int64_t o_b, int rows, int hidden, float eps, void* stream) {
  if (rows == 0) return MMP_OK;
  if (!x || !w || !out) return mmp_set_error(MMP_ERR_INVALID, "mmp_rmsnorm: null pointer");
  if (rows < 0 || hidden <= 0 || hidden % 8 || hidden > 256 * 8 * 8)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_rmsnorm: hidden %d must be a positive multiple of 8 <= 16384", hidden);
  if (!rows_ok(x, x_b) || !rows_ok(residual, r_b) || !rows_ok(sum_out, s_b) || !rows_ok(out, o_b) || !aligned16(w))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_rmsnorm: rows must be 16-byte aligned");
  RmsParams P{static_cast<const bf16*>(x), x_b, static_cast<const bf16*>(residual), r_b, static_cast<bf16*>(sum_out), s_b,
              static_cast<const bf16*>(w), static_cast<bf16*>(out), o_b, hidden, eps};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nvec = hidden / 8;
  if (nvec <= 256 * 2) { cudaError_t e = mmp::launch(rmsnorm_kernel<2>, dim3(rows), dim3(256), 0, s, nullptr, 0, P); if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_rmsnorm: %s", cudaGetErrorString(e)); }
  else if (nvec <= 256 * 4) { cudaError_t e = mmp::launch(rmsnorm_kernel<4>, dim3(rows), dim3(256), 0, s, nullptr, 0, P); if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_rmsnorm: %s", cudaGetErrorString(e)); }
  else { cudaError_t e = mmp::launch(rmsnorm_kernel<8>, dim3(rows), dim3(256), 0, s, nullptr, 0, P); if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_rmsnorm: %s", cudaGetErrorString(e)); }
  return mmp_check_launch("mmp_rmsnorm");
}

extern "C" int mmp_gated_rmsnorm(const void* y, int64_t y_b, const void* z, int64_t z_b, const void* w,
                                 void* out, int64_t o_b, float* sumsq, int rows, int D, int group_size,
                                 int mode, float count, float eps, void* stream) {
  if (rows == 0) return MMP_OK;
  if (!y || !z || (mode != 1 && (!w || !out)) || (mode != 0 && !sumsq))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gated_rmsnorm: null pointer");
  if (rows < 0 || rows > 65535 || D <= 0 || group_size <= 0 || D % group_size || group_size % 8 || group_size > 256 * 8 * 4 ||
      mode < 0 || mode > 3 || (mode == 2 && !(count > 0.f)))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gated_rmsnorm: bad sizes rows=%d D=%d group=%d mode=%d", rows, D, group_size, mode);
  if (!rows_ok(y, y_b) || !rows_ok(z, z_b) || (mode != 1 && (!rows_ok(out, o_b) || !aligned16(w))))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gated_rmsnorm: rows must be 16-byte aligned");
  GnParams P{static_cast<const bf16*>(y), y_b, static_cast<const bf16*>(z), z_b, static_cast<const bf16*>(w),
             static_cast<bf16*>(out), o_b, sumsq, D, group_size, mode, count, eps};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(D / group_size, rows);
  const int nvec = group_size / 8;
  if (nvec <= 256) { cudaError_t e = mmp::launch(gated_rmsnorm_kernel<1>, grid, dim3(256), 0, s, nullptr, 0, P); if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gated_rmsnorm: %s", cudaGetErrorString(e)); }
  else if (nvec <= 512) { cudaError_t e = mmp::launch(gated_rmsnorm_kernel<2>, grid, dim3(256), 0, s, nullptr, 0, P); if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gated_rmsnorm: %s", cudaGetErrorString(e)); }
  else { cudaError_t e = mmp::launch(gated_rmsnorm_kernel<4>, grid, dim3(256), 0, s, nullptr, 0, P); if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gated_rmsnorm: %s", cudaGetErrorString(e)); }
  return mmp_check_launch("mmp_gated_rmsnorm");
}

namespace mmp {
namespace {

__global__ void __launch_bounds__(256) silu_mul_kernel(const bf16* gate, int64_t g_b, const bf16* up, int64_t u_b,
                                                       bf16* out, int64_t o_b, int cols, float gs) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.y;
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= cols) return;
  float g[8], u[8], o[8];
  unpack8(ld16(gate + row * g_b + c0), g);
  unpack8(ld16(up + row * u_b + c0), u);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = silu(g[j] * gs) * u[j];
  st16(out + row * o_b + c0, pack8(o));
}

}  // namespace
}  // namespace mmp

extern "C" int mmp_silu_mul(const void* gate, int64_t g_b, const void* up, int64_t u_b, void* out, int64_t o_b,
                            int rows, int cols, float gate_scale, void* stream) {
  if (rows == 0 || cols == 0) return MMP_OK;
  if (!gate || !up || !out) return mmp_set_error(MMP_ERR_INVALID, "mmp_silu_mul: null pointer");
  if (rows < 0 || rows > 65535 || cols < 0 || cols % 8 || !rows_ok(gate, g_b) || !rows_ok(up, u_b) || !rows_ok(out, o_b))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_silu_mul: cols %% 8 == 0 and 16-byte aligned rows required");
  dim3 grid((cols / 8 + 255) / 256, rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = mmp::launch(silu_mul_kernel, grid, dim3(256), 0, s, nullptr, 0, static_cast<const bf16*>(gate), g_b,
                              static_cast<const bf16*>(up), u_b, static_cast<bf16*>(out), o_b, cols, gate_scale);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_silu_mul: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_silu_mul");
}

namespace mmp {
namespace {

__global__ void __launch_bounds__(256) add3_kernel(const bf16* a, int64_t a_b, const bf16* b, int64_t b_b, const bf16* c,
                                                   int64_t c_b, bf16* out, int64_t o_b, int cols) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.y;
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= cols) return;
  float x[8], y[8];
  unpack8(ld16(a + row * a_b + c0), x);
  unpack8(ld16(b + row * b_b + c0), y);
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] += y[j];
  if (c) {
    unpack8(ld16(c + row * c_b + c0), y);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] += y[j];
  }
  st16(out + row * o_b + c0, pack8(x));
}

}  // namespace
}  // namespace mmp

extern "C" int mmp_add(const void* a, int64_t a_b, const void* b, int64_t b_b, const void* c, int64_t c_b,
                       void* out, int64_t o_b, int rows, int cols, void* stream) {
  if (rows == 0 || cols == 0) return MMP_OK;
  if (!a || !b || !out) return mmp_set_error(MMP_ERR_INVALID, "mmp_add: null pointer");
  if (rows < 0 || rows > 65535 || cols < 0 || cols % 8 || !rows_ok(a, a_b) || !rows_ok(b, b_b) || !rows_ok(c, c_b) ||
      !rows_ok(out, o_b))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_add: cols %% 8 == 0 and 16-byte aligned rows required");
  dim3 grid((cols / 8 + 255) / 256, rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = mmp::launch(add3_kernel, grid, dim3(256), 0, s, nullptr, 0, static_cast<const bf16*>(a), a_b,
                              static_cast<const bf16*>(b), b_b, static_cast<const bf16*>(c), c_b, static_cast<bf16*>(out),
                              o_b, cols);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_add: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_add");
}

extern "C" int mmp_scale_rows(void* x, int64_t ld, const float* sumsq, int rows, int cols, float count, float eps,
                              void* stream) {
  if (rows == 0 || cols == 0) return MMP_OK;
  if (!x || !sumsq) return mmp_set_error(MMP_ERR_INVALID, "mmp_scale_rows: null pointer");
  if (rows < 0 || rows > 65535 || cols < 0 || cols % 8 || !(count > 0.f) || !rows_ok(x, ld))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_scale_rows: rows=%d cols=%d (multiple of 8), 16-byte aligned rows", rows,
                         cols);
  cudaError_t e = mmp::launch(scale_rows_kernel, dim3(rows), dim3(256), 0, static_cast<cudaStream_t>(stream), nullptr, 0,
                              static_cast<bf16*>(x), ld, sumsq, cols, count, eps);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_scale_rows: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_scale_rows");
}
