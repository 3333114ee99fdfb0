// Causal GQA attention for prefill over the paged KV cache (FlashAttention-2 varlen with causal=True in the
// serving stack the reference measures; the reference harness itself only decodes).
//
// Query token j of sequence i sits at position ctx_start[i] + j and attends to cache positions
// [0, ctx_start[i] + j] of that sequence (the new tokens' keys/values are already in the cache), so the same
// kernel serves prefill from scratch (ctx_start = 0) and chunked prefill over cached context. CTA = 128 query
// tokens of one query head; 4 warps x two 16-row m-tiles (each K/V fragment feeds both); K/V tiles of 64 tokens gathered page by page from the
// cache into a double-buffered cp.async ring; S = Q K^T and O += P V on mma.m16n8k16 (bf16 in, fp32
// accumulate) with an online softmax in the exp2 domain.
#include <algorithm>

#include "mmp_common.cuh"

namespace mmp {
namespace {

constexpr int MT = 2;                       // 16-row m-tiles per warp
constexpr int NW = 4;                       // warps
constexpr int BQ = 16 * MT * NW, BKV = 64, HD = 128, ATHR = 32 * NW;
constexpr int ROWB = HD * 2;  // bytes per K/V/Q row

struct AttnPrefillParams {
  const bf16* q; int64_t q_t, q_h;
  const bf16* kc; const bf16* vc; int64_t c_block, c_tok, c_head;
  const int32_t* block_table; int64_t bt_stride;
  const int32_t* cu_q;
  const int32_t* ctx_start;
  bf16* out; int64_t o_t, o_h;
  int nq, nkv, block_size, num_blocks;
  int block_shift;  // log2(block_size) when it is a power of two, else -1
  float scale_log2;
  int* err;
};

__device__ __forceinline__ uint32_t sa(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * ROWB + ((c ^ (r & 7)) << 4); }
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
__device__ __forceinline__ float ex2(float x) {  // 2^x on the MUFU unit (ex2.approx.ftz; 2^-inf = 0)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}

constexpr int Q_OFF = 0, K_OFF = BQ * ROWB, V_OFF = K_OFF + 2 * BKV * ROWB, SMEM = V_OFF + 2 * BKV * ROWB;

// grid (nq, nseq, q tiles): tile index from the slowest dimension, reversed, so the CTAs with the longest key
// ranges (last query tiles) start first and the short ones fill the tail.
__global__ void __launch_bounds__(ATHR, 2) attn_prefill_kernel(const AttnPrefillParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_trigger();
  pdl_wait();
  const int head = blockIdx.x, seq = blockIdx.y, j0 = (gridDim.z - 1 - blockIdx.z) * BQ;
  const int q0 = P.cu_q[seq], qlen = P.cu_q[seq + 1] - q0;
  if (j0 >= qlen) return;
  const int start = P.ctx_start[seq];
  const int kh = head / (P.nq / P.nkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const uint32_t base = sa(smem);
  const int j_last = min(j0 + BQ - 1, qlen - 1);
  const int total = start + qlen;               // keys of the sequence
  const int kend = start + j_last + 1;          // keys any row of this tile can see
  const int nkt = (kend + BKV - 1) / BKV;

  // Q tile
  for (int i = tid; i < BQ * (ROWB / 16); i += ATHR) {
    const int r = i / (ROWB / 16), c = i % (ROWB / 16);
    const bool v = j0 + r < qlen;
    cp16(base + Q_OFF + swz(r, c), P.q + static_cast<int64_t>(q0 + (v ? j0 + r : 0)) * P.q_t + head * P.q_h + c * 8, v);
  }
  // K/V tile rows: thread t copies 16-byte chunk (t % 16) of rows t / 16 + 8 n
  const int kv_c = tid % (ROWB / 16), kv_r0 = tid / (ROWB / 16);
  constexpr int KV_ROWS_PER_PASS = ATHR / (ROWB / 16);
  const int32_t* btab = P.block_table + static_cast<int64_t>(seq) * P.bt_stride;
  const int64_t head_off = kh * P.c_head + kv_c * 8;
  auto issue_kv = [&](int kt, int stage) {
#pragma unroll
    for (int n = 0; n < BKV / KV_ROWS_PER_PASS; ++n) {
      const int r = kv_r0 + n * KV_ROWS_PER_PASS;
      const int tok = kt * BKV + r;
      int blk = -1, in_blk = 0;
      if (tok < total) {
        int col;
        if (P.block_shift >= 0) {
          col = tok >> P.block_shift;
          in_blk = tok & (P.block_size - 1);
        } else {
          col = tok / P.block_size;
          in_blk = tok - col * P.block_size;
        }
        blk = col < P.bt_stride ? __ldg(btab + col) : -1;
        if (blk < 0 || blk >= P.num_blocks) {
          flag_error(P.err, DEVERR_INDEX);
          blk = -1;
        }
      }
      const int64_t off = blk < 0 ? 0 : blk * P.c_block + in_blk * P.c_tok + head_off;
      cp16(base + K_OFF + stage * BKV * ROWB + swz(r, kv_c), P.kc + off, blk >= 0);
      cp16(base + V_OFF + stage * BKV * ROWB + swz(r, kv_c), P.vc + off, blk >= 0);
    }
  };
  issue_kv(0, 0);
  asm volatile("cp.async.commit_group;\n" ::);

  // this warp's query rows: m-tile i covers tile rows warp*16 + i*64 .. +15; lane rows g and g + 8
  const int warp_first = start + j0 + warp * 16;  // smallest query position of the warp
  const int warp_kend = start + min(j0 + warp * 16 + (MT - 1) * 16 * NW + 15, qlen - 1) + 1;
  float o[MT][HD / 8][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) o[i][n][0] = o[i][n][1] = o[i][n][2] = o[i][n][3] = 0.f;
  float m[MT][2], l[MT][2];
#pragma unroll
  for (int i = 0; i < MT; ++i) m[i][0] = m[i][1] = -INFINITY, l[i][0] = l[i][1] = 0.f;
  const int mat = lane >> 3, r8 = lane & 7;
  const float sc = P.scale_log2;

  for (int kt = 0; kt < nkt; ++kt) {
    if (kt + 1 < nkt) issue_kv(kt + 1, (kt + 1) & 1);
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 1;\n" ::);
    __syncthreads();
    const int k0 = kt * BKV;
    if (k0 < warp_kend) {
      const uint32_t sK = base + K_OFF + (kt & 1) * BKV * ROWB, sV = base + V_OFF + (kt & 1) * BKV * ROWB;
      float s[MT][BKV / 8][4];
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int n = 0; n < BKV / 8; ++n) s[i][n][0] = s[i][n][1] = s[i][n][2] = s[i][n][3] = 0.f;
#pragma unroll
      for (int k = 0; k < HD / 16; ++k) {
        uint32_t qf[MT][4];
#pragma unroll
        for (int i = 0; i < MT; ++i)
          ldsm_x4(base + Q_OFF + swz(warp * 16 + i * 16 * NW + (mat & 1) * 8 + r8, k * 2 + (mat >> 1)), qf[i]);
#pragma unroll
        for (int np = 0; np < BKV / 16; ++np) {
          uint32_t b[4];
          ldsm_x4(sK + swz(np * 16 + (mat >> 1) * 8 + r8, k * 2 + (mat & 1)), b);
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            mma16816(s[i][2 * np], qf[i], b[0], b[1]);
            mma16816(s[i][2 * np + 1], qf[i], b[2], b[3]);
          }
        }
      }
      // a tile wholly inside every row's visible range needs no mask
      const bool full = k0 + BKV - 1 <= warp_first && k0 + BKV <= total;
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < BKV / 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int kp = k0 + nt * 8 + 2 * tq + (e & 1);
            const int qp = warp_first + i * 16 * NW + g + (e >> 1) * 8;
            if (!full && !(kp <= qp && kp < total)) s[i][nt][e] = -INFINITY;
          }
          mx0 = fmaxf(mx0, fmaxf(s[i][nt][0], s[i][nt][1]));
          mx1 = fmaxf(mx1, fmaxf(s[i][nt][2], s[i][nt][3]));
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        // running maxima are kept on raw scores; p = 2^(s * scale_log2 - m * scale_log2) is one FFMA + ex2
        const float mn0 = fmaxf(m[i][0], mx0), mn1 = fmaxf(m[i][1], mx1);
        // rows with nothing visible yet keep a zero base so the exponent stays finite
        const float b0 = mn0 == -INFINITY ? 0.f : mn0 * sc, b1 = mn1 == -INFINITY ? 0.f : mn1 * sc;
        const float al0 = ex2(fmaf(m[i][0], sc, -b0)), al1 = ex2(fmaf(m[i][1], sc, -b1));
        m[i][0] = mn0;
        m[i][1] = mn1;
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < BKV / 8; ++nt) {
          s[i][nt][0] = ex2(fmaf(s[i][nt][0], sc, -b0));
          s[i][nt][1] = ex2(fmaf(s[i][nt][1], sc, -b0));
          s[i][nt][2] = ex2(fmaf(s[i][nt][2], sc, -b1));
          s[i][nt][3] = ex2(fmaf(s[i][nt][3], sc, -b1));
          sum0 += s[i][nt][0] + s[i][nt][1];
          sum1 += s[i][nt][2] + s[i][nt][3];
        }
        l[i][0] = l[i][0] * al0 + sum0;
        l[i][1] = l[i][1] * al1 + sum1;
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) {
          o[i][n][0] *= al0;
          o[i][n][1] *= al0;
          o[i][n][2] *= al1;
          o[i][n][3] *= al1;
        }
      }
#pragma unroll
      for (int kk = 0; kk < BKV / 16; ++kk) {  // O += P V, K = keys
        uint32_t a[MT][4];
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          a[i][0] = pack_bf16x2(s[i][2 * kk][0], s[i][2 * kk][1]);
          a[i][1] = pack_bf16x2(s[i][2 * kk][2], s[i][2 * kk][3]);
          a[i][2] = pack_bf16x2(s[i][2 * kk + 1][0], s[i][2 * kk + 1][1]);
          a[i][3] = pack_bf16x2(s[i][2 * kk + 1][2], s[i][2 * kk + 1][3]);
        }
#pragma unroll
        for (int np = 0; np < HD / 16; ++np) {
          uint32_t b[4];  // V[key][d]: transposed load gives (k = key, n = d) fragments for d-tiles 2np, 2np + 1
          ldsm_x4_t(sV + swz(kk * 16 + (mat & 1) * 8 + r8, np * 2 + (mat >> 1)), b);
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            mma16816(o[i][2 * np], a[i], b[0], b[1]);
            mma16816(o[i][2 * np + 1], a[i], b[2], b[3]);
          }
        }
      }
    }
    __syncthreads();  // this stage is refilled two iterations from now
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
#pragma unroll
  for (int i = 0; i < MT; ++i) {
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      l[i][0] += __shfl_xor_sync(0xffffffffu, l[i][0], off);
      l[i][1] += __shfl_xor_sync(0xffffffffu, l[i][1], off);
    }
    const float inv0 = l[i][0] > 0.f ? 1.f / l[i][0] : 0.f, inv1 = l[i][1] > 0.f ? 1.f / l[i][1] : 0.f;
    const int jr0 = j0 + warp * 16 + i * 16 * NW + g, jr1 = jr0 + 8;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt) {
      const int d = nt * 8 + 2 * tq;
      if (jr0 < qlen)
        *reinterpret_cast<uint32_t*>(P.out + static_cast<int64_t>(q0 + jr0) * P.o_t + head * P.o_h + d) =
            pack_bf16x2(o[i][nt][0] * inv0, o[i][nt][1] * inv0);
      if (jr1 < qlen)
        *reinterpret_cast<uint32_t*>(P.out + static_cast<int64_t>(q0 + jr1) * P.o_t + head * P.o_h + d) =
            pack_bf16x2(o[i][nt][2] * inv1, o[i][nt][3] * inv1);
    }
  }
}

}  // namespace

int attn_prefill_tc(const void* q, int64_t q_t, int64_t q_h, const void* key_cache, const void* value_cache,
                    int64_t c_block, int64_t c_tok, int64_t c_head, const int32_t* block_table, int64_t bt_stride,
                    const int32_t* cu_q, const int32_t* ctx_start, void* out, int64_t o_t, int64_t o_h, int nseq,
                    int max_q_len, int nq, int nkv, int hd, int block_size, int num_blocks, float scale, int* err,
                    cudaStream_t stream);
}  // namespace mmp

using namespace mmp;

extern "C" int mmp_paged_attn_prefill(const void* q, int64_t q_t, int64_t q_h,
                                      const void* key_cache, const void* value_cache, int64_t c_block, int64_t c_tok,
                                      int64_t c_head, const int32_t* block_table, int64_t bt_stride,
                                      const int32_t* cu_q, const int32_t* ctx_start, void* out, int64_t o_t, int64_t o_h,
                                      int nseq, int max_q_len, int nq, int nkv, int hd, int block_size, int num_blocks,
                                      float scale, int* err, void* stream) {
  if (nseq == 0 || max_q_len == 0) return MMP_OK;
  if (!q || !key_cache || !value_cache || !block_table || !cu_q || !ctx_start || !out)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_paged_attn_prefill: null pointer");
  if (hd != HD) return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_paged_attn_prefill: head_dim %d (only 128)", hd);
  if (nseq < 0 || nseq > 65535 || max_q_len < 0 || nq <= 0 || nq > 65535 || nkv <= 0 || nq % nkv || block_size <= 0 ||
      num_blocks <= 0)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_paged_attn_prefill: bad sizes");
  if (!aligned16(q) || !aligned16(key_cache) || !aligned16(value_cache) || q_t % 8 || q_h % 8 || c_block % 8 ||
      c_tok % 8 || c_head % 8 || (o_t | o_h) & 1 || (reinterpret_cast<uintptr_t>(out) & 3))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_paged_attn_prefill: q and cache rows must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    const int rc = attn_prefill_tc(q, q_t, q_h, key_cache, value_cache, c_block, c_tok, c_head, block_table, bt_stride,
                                   cu_q, ctx_start, out, o_t, o_h, nseq, max_q_len, nq, nkv, hd, block_size, num_blocks,
                                   scale, err, s);
    if (rc != MMP_ERR_UNSUPPORTED) return rc;  // ran on the tensor cores (or failed there)
  }
  AttnPrefillParams P{static_cast<const bf16*>(q), q_t, q_h, static_cast<const bf16*>(key_cache),
                      static_cast<const bf16*>(value_cache), c_block, c_tok, c_head, block_table, bt_stride, cu_q,
                      ctx_start, static_cast<bf16*>(out), o_t, o_h, nq, nkv, block_size, num_blocks,
                      (block_size & (block_size - 1)) == 0 ? __builtin_ctz(block_size) : -1,
                      scale * 1.4426950408889634f, err};
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_prefill: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  const int tiles = (max_q_len + BQ - 1) / BQ;
  if (tiles > 65535) return mmp_set_error(MMP_ERR_INVALID, "mmp_paged_attn_prefill: max_q_len too large");
  dim3 grid(nq, nseq, tiles);
  cudaError_t e = mmp::launch(attn_prefill_kernel, grid, dim3(ATHR), SMEM, s, nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_prefill: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_paged_attn_prefill");
}
