// Causal GQA attention for prefill over the paged KV cache (FlashAttention-2 varlen with causal=True in the
// serving stack the reference measures; the reference harness itself only decodes).
//
// Query token j of sequence i sits at position ctx_start[i] + j and attends to cache positions
// [0, ctx_start[i] + j] of that sequence (the new tokens' keys/values are already in the cache), so the same
// kernel serves prefill from scratch (ctx_start = 0) and chunked prefill over cached context. CTA = 64 query
// tokens of one query head; 4 warps x 16 query rows; K/V tiles of 64 tokens gathered page by page from the
// cache into a double-buffered cp.async ring; S = Q K^T and O += P V on mma.m16n8k16 (bf16 in, fp32
// accumulate) with an online softmax in the exp2 domain.
#include <algorithm>

#include "mmp_common.cuh"

namespace mmp {
namespace {

constexpr int BQ = 64, BKV = 64, HD = 128, ATHR = 128;
constexpr int ROWB = HD * 2;  // bytes per K/V/Q row

struct AttnPrefillParams {
  const bf16* q; int64_t q_t, q_h;
  const bf16* kc; const bf16* vc; int64_t c_block, c_tok, c_head;
  const int32_t* block_table; int64_t bt_stride;
  const int32_t* cu_q;
  const int32_t* ctx_start;
  bf16* out; int64_t o_t, o_h;
  int nq, nkv, block_size, num_blocks;
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
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}

constexpr int Q_OFF = 0, K_OFF = BQ * ROWB, V_OFF = K_OFF + 2 * BKV * ROWB, SMEM = V_OFF + 2 * BKV * ROWB;

__global__ void __launch_bounds__(ATHR) attn_prefill_kernel(const AttnPrefillParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_trigger();
  pdl_wait();
  const int j0 = blockIdx.x * BQ, head = blockIdx.y, seq = blockIdx.z;
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
  auto issue_kv = [&](int kt, int stage) {
    for (int i = tid; i < BKV * (ROWB / 16); i += ATHR) {
      const int r = i / (ROWB / 16), c = i % (ROWB / 16);
      const int tok = kt * BKV + r;
      int blk = -1;
      if (tok < total) {
        const int col = tok / P.block_size;
        blk = col < P.bt_stride ? P.block_table[seq * P.bt_stride + col] : -1;
        if (blk < 0 || blk >= P.num_blocks) {
          flag_error(P.err, DEVERR_INDEX);
          blk = -1;
        }
      }
      const int64_t off = blk < 0 ? 0 : blk * P.c_block + (tok % P.block_size) * P.c_tok + kh * P.c_head + c * 8;
      cp16(base + K_OFF + stage * BKV * ROWB + swz(r, c), P.kc + off, blk >= 0);
      cp16(base + V_OFF + stage * BKV * ROWB + swz(r, c), P.vc + off, blk >= 0);
    }
  };
  issue_kv(0, 0);
  asm volatile("cp.async.commit_group;\n" ::);

  const int r0 = warp * 16;                       // this warp's 16 query rows
  const int qpos_lo = start + j0 + r0 + g;        // positions of rows g and g+8
  const int qpos_hi = qpos_lo + 8;
  const int warp_kend = start + min(j0 + r0 + 15, qlen - 1) + 1;
  uint32_t qf[HD / 16][4];
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  const int mat = lane >> 3, r8 = lane & 7;

  for (int kt = 0; kt < nkt; ++kt) {
    if (kt + 1 < nkt) issue_kv(kt + 1, (kt + 1) & 1);
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 1;\n" ::);
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int k = 0; k < HD / 16; ++k) ldsm_x4(base + Q_OFF + swz(r0 + (mat & 1) * 8 + r8, k * 2 + (mat >> 1)), qf[k]);
    }
    const int k0 = kt * BKV;
    if (k0 < warp_kend) {
      const uint32_t sK = base + K_OFF + (kt & 1) * BKV * ROWB, sV = base + V_OFF + (kt & 1) * BKV * ROWB;
      float s[BKV / 8][4];
#pragma unroll
      for (int i = 0; i < BKV / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
      for (int k = 0; k < HD / 16; ++k) {
#pragma unroll
        for (int np = 0; np < BKV / 16; ++np) {
          uint32_t b[4];
          ldsm_x4(sK + swz(np * 16 + (mat >> 1) * 8 + r8, k * 2 + (mat & 1)), b);
          mma16816(s[2 * np], qf[k], b[0], b[1]);
          mma16816(s[2 * np + 1], qf[k], b[2], b[3]);
        }
      }
      float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < BKV / 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kp = k0 + nt * 8 + 2 * tq + (e & 1);
          const int qp = e < 2 ? qpos_lo : qpos_hi;
          s[nt][e] = (kp <= qp && kp < total) ? s[nt][e] * P.scale_log2 : -INFINITY;
        }
        mx_lo = fmaxf(mx_lo, fmaxf(s[nt][0], s[nt][1]));
        mx_hi = fmaxf(mx_hi, fmaxf(s[nt][2], s[nt][3]));
      }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
        mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
      }
      const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
      // rows with nothing visible yet keep a zero base so exp2 stays finite
      const float b_lo = mn_lo == -INFINITY ? 0.f : mn_lo, b_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
      const float al_lo = exp2f(m_lo - b_lo), al_hi = exp2f(m_hi - b_hi);
      m_lo = mn_lo;
      m_hi = mn_hi;
      float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
      for (int nt = 0; nt < BKV / 8; ++nt) {
        s[nt][0] = exp2f(s[nt][0] - b_lo);
        s[nt][1] = exp2f(s[nt][1] - b_lo);
        s[nt][2] = exp2f(s[nt][2] - b_hi);
        s[nt][3] = exp2f(s[nt][3] - b_hi);
        sum_lo += s[nt][0] + s[nt][1];
        sum_hi += s[nt][2] + s[nt][3];
      }
      l_lo = l_lo * al_lo + sum_lo;
      l_hi = l_hi * al_hi + sum_hi;
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) {
        o[i][0] *= al_lo;
        o[i][1] *= al_lo;
        o[i][2] *= al_hi;
        o[i][3] *= al_hi;
      }
#pragma unroll
      for (int kk = 0; kk < BKV / 16; ++kk) {  // O += P V, K = keys
        uint32_t a[4];
        a[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
        a[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
        a[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        a[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int np = 0; np < HD / 16; ++np) {
          uint32_t b[4];  // V[key][d]: transposed load gives (k = key, n = d) fragments for d-tiles 2np, 2np + 1
          ldsm_x4_t(sV + swz(kk * 16 + (mat & 1) * 8 + r8, np * 2 + (mat >> 1)), b);
          mma16816(o[2 * np], a, b[0], b[1]);
          mma16816(o[2 * np + 1], a, b[2], b[3]);
        }
      }
    }
    __syncthreads();  // this stage is refilled two iterations from now
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
  }
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f, inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  const int jr_lo = j0 + r0 + g, jr_hi = jr_lo + 8;
#pragma unroll
  for (int nt = 0; nt < HD / 8; ++nt) {
    const int d = nt * 8 + 2 * tq;
    if (jr_lo < qlen)
      *reinterpret_cast<uint32_t*>(P.out + static_cast<int64_t>(q0 + jr_lo) * P.o_t + head * P.o_h + d) =
          pack_bf16x2(o[nt][0] * inv_lo, o[nt][1] * inv_lo);
    if (jr_hi < qlen)
      *reinterpret_cast<uint32_t*>(P.out + static_cast<int64_t>(q0 + jr_hi) * P.o_t + head * P.o_h + d) =
          pack_bf16x2(o[nt][2] * inv_hi, o[nt][3] * inv_hi);
  }
}

}  // namespace
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
  AttnPrefillParams P{static_cast<const bf16*>(q), q_t, q_h, static_cast<const bf16*>(key_cache),
                      static_cast<const bf16*>(value_cache), c_block, c_tok, c_head, block_table, bt_stride, cu_q,
                      ctx_start, static_cast<bf16*>(out), o_t, o_h, nq, nkv, block_size, num_blocks,
                      scale * 1.4426950408889634f, err};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_prefill: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  dim3 grid((max_q_len + BQ - 1) / BQ, nq, nseq);
  cudaError_t e = mmp::launch(attn_prefill_kernel, grid, dim3(ATHR), SMEM, s, nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_prefill: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_paged_attn_prefill");
}
