// bf16 GEMM out = alpha * colscale .* (A W^T) + addend for the layer's projections (replaces F.linear / @
// and the scalings the reference layer applies to their results, harness/kernels.py:147-154 and
// harness/layer.py:35,80,105).
//
// Decode shapes (M = batch <= 256) are weight-streaming: the kernel must keep HBM busy reading W once.
// CTA tile 64 x 64 x 64, 4 warps (2 x 2, 32 x 32 each), 4-stage cp.async pipeline into 128-byte-swizzled
// shared memory, ldmatrix + mma.m16n8k16. When there are too few output tiles to fill the GPU, K is
// split over the CTAs of a thread-block cluster (up to 8) and the fp32 partial tiles are summed through
// distributed shared memory by the cluster itself: no global workspace and no second launch.
#include <algorithm>
#include <cooperative_groups.h>

#include "mmp_common.cuh"

namespace cg = cooperative_groups;

namespace mmp {
namespace {

constexpr int BM = 64, BN = 64, BK = 64, STAGES = 4, THREADS = 128;
constexpr int TILE_BYTES = BM * BK * 2;  // == BN * BK * 2
constexpr int SMEM_BYTES = STAGES * 2 * TILE_BYTES;
constexpr int RED_LD = BN + 4;  // padded fp32 row of the partial tile

struct GemmParams {
  const bf16* a; int64_t lda;
  const bf16* w; int64_t ldw;
  bf16* out; int64_t ldo;
  const float* colscale;
  const bf16* addend; int64_t ldd;
  int M, N, K;
  float alpha;
  int k_tiles_per_split;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// byte offset of 16-byte chunk `chunk` of row `row` in a [rows][64] bf16 tile with a 128-byte XOR swizzle
__device__ __forceinline__ uint32_t swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ void load_stage(const GemmParams& P, uint32_t sA, uint32_t sW, int m0, int n0, int k0,
                                           int k_end) {
#pragma unroll
  for (int i = 0; i < (BM * BK / 8) / THREADS; ++i) {
    const int c = threadIdx.x + i * THREADS;
    const int row = c >> 3, ch = c & 7;
    const int k = k0 + ch * 8;
    const bool va = (m0 + row < P.M) && (k < k_end);
    const bf16* ga = va ? P.a + static_cast<int64_t>(m0 + row) * P.lda + k : P.a;
    cp_async16(sA + swz(row, ch), ga, va);
    const bool vw = (n0 + row < P.N) && (k < k_end);
    const bf16* gw = vw ? P.w + static_cast<int64_t>(n0 + row) * P.ldw + k : P.w;
    cp_async16(sW + swz(row, ch), gw, vw);
  }
}

__device__ __forceinline__ float epilogue_value(const GemmParams& P, float acc, int row, int col) {
  float v = acc * P.alpha;
  if (P.colscale) v *= P.colscale[col];
  if (P.addend) v += bf2f(P.addend[static_cast<int64_t>(row) * P.ldd + col]);
  return v;
}

__device__ __forceinline__ void store_pair(const GemmParams& P, int row, int col, float v0, float v1) {
  if (row >= P.M || col >= P.N) return;
  bf16* dst = P.out + static_cast<int64_t>(row) * P.ldo + col;
  const float a = epilogue_value(P, v0, row, col);
  if (col + 1 < P.N) {
    const float b = epilogue_value(P, v1, row, col + 1);
    if ((reinterpret_cast<uintptr_t>(dst) & 3u) == 0) {
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(a, b);
    } else {
      dst[0] = f2bf(a);
      dst[1] = f2bf(b);
    }
  } else {
    dst[0] = f2bf(a);
  }
}

template <bool CLUSTER>
__global__ void __launch_bounds__(THREADS) gemm_bf16_kernel(const GemmParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int split = blockIdx.z;
  const int k_tiles_total = (P.K + BK - 1) / BK;
  const int kt0 = split * P.k_tiles_per_split;
  const int kt1 = min(k_tiles_total, kt0 + P.k_tiles_per_split);
  const int nkt = max(0, kt1 - kt0);
  const int k_end = min(P.K, kt1 * BK);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wm = warp >> 1, wn = warp & 1;
  const uint32_t base = smem_u32(smem);
  auto sA = [&](int s) { return base + s * 2 * TILE_BYTES; };
  auto sW = [&](int s) { return base + s * 2 * TILE_BYTES + TILE_BYTES; };

  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < nkt) load_stage(P, sA(s), sW(s), m0, n0, (kt0 + s) * BK, k_end);
    cp_async_commit();
  }
  for (int it = 0; it < nkt; ++it) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    const int nxt = it + STAGES - 1;
    if (nxt < nkt) load_stage(P, sA(nxt % STAGES), sW(nxt % STAGES), m0, n0, (kt0 + nxt) * BK, k_end);
    cp_async_commit();
    const uint32_t a_s = sA(it % STAGES), w_s = sW(it % STAGES);
#pragma unroll
    for (int ks = 0; ks < BK / 16; ++ks) {
      uint32_t af[2][4], bfr[4][2];
      const int mat = lane >> 3, r8 = lane & 7;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int row = wm * 32 + mt * 16 + (mat & 1) * 8 + r8;
        ldmatrix_x4(a_s + swz(row, ks * 2 + (mat >> 1)), af[mt][0], af[mt][1], af[mt][2], af[mt][3]);
      }
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int row = wn * 32 + np * 16 + (mat >> 1) * 8 + r8;
        ldmatrix_x4(w_s + swz(row, ks * 2 + (mat & 1)), bfr[2 * np][0], bfr[2 * np][1], bfr[2 * np + 1][0],
                    bfr[2 * np + 1][1]);
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma16816(acc[mt][nt], af[mt], bfr[nt][0], bfr[nt][1]);
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  const int g = lane >> 2, t = lane & 3;
  if constexpr (!CLUSTER) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int row = m0 + wm * 32 + mt * 16 + g;
        const int col = n0 + wn * 32 + nt * 8 + 2 * t;
        store_pair(P, row, col, acc[mt][nt][0], acc[mt][nt][1]);
        store_pair(P, row + 8, col, acc[mt][nt][2], acc[mt][nt][3]);
      }
  } else {
    // split-K: park the fp32 partial tile in this CTA's shared memory, then every CTA of the cluster sums
    // its share of the rows over all CTAs' tiles through distributed shared memory.
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int r = wm * 32 + mt * 16 + g, c = wn * 32 + nt * 8 + 2 * t;
        *reinterpret_cast<float2*>(&red[r * RED_LD + c]) = make_float2(acc[mt][nt][0], acc[mt][nt][1]);
        *reinterpret_cast<float2*>(&red[(r + 8) * RED_LD + c]) = make_float2(acc[mt][nt][2], acc[mt][nt][3]);
      }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int nsplit = static_cast<int>(cluster.num_blocks());
    const int me = static_cast<int>(cluster.block_rank());
    const int rows_per = (BM + nsplit - 1) / nsplit;
    const int r_lo = me * rows_per, r_hi = min(BM, r_lo + rows_per);
    for (int idx = threadIdx.x; idx < (r_hi - r_lo) * (BN / 2); idx += THREADS) {
      const int r = r_lo + idx / (BN / 2), c = (idx % (BN / 2)) * 2;
      float2 sum = make_float2(0.f, 0.f);
      for (int q = 0; q < nsplit; ++q) {
        const float* rem = cluster.map_shared_rank(red, q);
        const float2 v = *reinterpret_cast<const float2*>(&rem[r * RED_LD + c]);
        sum.x += v.x;
        sum.y += v.y;
      }
      store_pair(P, m0 + r, n0 + c, sum.x, sum.y);
    }
    cluster.sync();
  }
}

int g_sms = 0;
bool g_attr_set[2] = {false, false};

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" int mmp_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int64_t ldo,
                             int M, int N, int K, float alpha, const float* colscale, const void* addend, int64_t ldd,
                             void* stream) {
  if (M == 0 || N == 0) return MMP_OK;
  if (!a || !w || !out) return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16: null pointer");
  if (M < 0 || N < 0 || K <= 0 || K % 8 || lda % 8 || ldw % 8 || !aligned16(a) || !aligned16(w) || lda < K || ldw < K ||
      ldo < N || (addend && ldd < N))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16: M=%d N=%d K=%d lda=%lld ldw=%lld: K and strides must be "
                         "multiples of 8 with 16-byte aligned bases", M, N, K, (long long)lda, (long long)ldw);
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms <= 0) g_sms = 148;
  }
  const int tiles_n = (N + BN - 1) / BN, tiles_m = (M + BM - 1) / BM;
  if (tiles_m > 65535) return mmp_set_error(MMP_ERR_INVALID, "mmp_gemm_bf16: M=%d too large", M);
  const int k_tiles = (K + BK - 1) / BK;
  const int tiles = tiles_n * tiles_m;
  int split = 1;
  if (tiles < 2 * g_sms) {
    split = (2 * g_sms + tiles - 1) / tiles;
    split = std::min(split, std::max(1, k_tiles / 2));
    split = std::min(split, 8);
  }
  const int ktps = (k_tiles + split - 1) / split;
  split = (k_tiles + ktps - 1) / ktps;
  GemmParams P{static_cast<const bf16*>(a), lda, static_cast<const bf16*>(w), ldw, static_cast<bf16*>(out), ldo,
               colscale, static_cast<const bf16*>(addend), ldd, M, N, K, alpha, ktps};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles_n, tiles_m, split);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  cudaError_t e;
  if (split > 1) {
    if (!g_attr_set[1]) {
      cudaFuncSetAttribute(gemm_bf16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
      g_attr_set[1] = true;
    }
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = split;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<true>, P);
  } else {
    if (!g_attr_set[0]) {
      cudaFuncSetAttribute(gemm_bf16_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
      g_attr_set[0] = true;
    }
    e = cudaLaunchKernelEx(&cfg, gemm_bf16_kernel<false>, P);
  }
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gemm_bf16: launch failed: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_gemm_bf16");
}
