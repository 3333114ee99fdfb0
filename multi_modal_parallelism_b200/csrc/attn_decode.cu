// Paged GQA decode attention, one query token per sequence (replaces FlashAttention-2 varlen with
// max_seqlen_q = 1 as called by harness/kernels.py:118-127 of the reference).
//
// HBM-bound: every key/value of every sequence is read once. Work split: CTA = (key range "split", KV
// head, sequence); its 4 warps take 16-token tiles of the range in turn. A tile's keys and values go from
// HBM straight into mma fragments (16-byte loads; the head dimension is permuted consistently between the
// query and key fragments so each lane reads 16 contiguous bytes of a key row; values are transposed in
// registers with movmatrix). Scores and P.V use mma.m16n8k16 bf16 -> fp32 with the <= 16 query heads of
// the KV head as the M rows. Online softmax in the exp2 domain. Warps merge in shared memory; splits
// merge through the workspace in a second kernel (log-sum-exp weighting).
#include <algorithm>

#include "mmp_common.cuh"

namespace mmp {
namespace {

constexpr int TILE = 16;   // tokens per mma tile
constexpr int WARPS = 4;

struct AttnParams {
  const bf16* q; int64_t q_b, q_h;
  const bf16* kc; const bf16* vc; int64_t c_block, c_tok, c_head;
  const int32_t* block_table; int64_t bt_stride;
  const int32_t* seqlens;
  bf16* out; int64_t o_b, o_h;
  float* part_o;   // [batch, nq, splits, HD]
  float* part_ml;  // [batch, nq, splits, 2]
  int batch, nq, nkv, block_size, num_blocks, splits, tiles_per_split;
  float scale_log2;
  int* err;
};

__device__ __forceinline__ void mma_bf16_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t transpose8x8(uint32_t v) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(r) : "r"(v));
  return r;
}

__device__ __forceinline__ uint32_t word(const uint4& u, int j) {
  return j == 0 ? u.x : j == 1 ? u.y : j == 2 ? u.z : u.w;
}

constexpr int STAGES = 3;           // pages in flight per warp
constexpr int PAGE_BYTES = TILE * 512; // 16 tokens x (128 keys + 128 values) x bf16

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }
__device__ __forceinline__ uint4 lds16(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
// byte offset of 16-byte chunk c (0..15 keys, 16..31 values) of token row r inside a page; rows r and r^1 use
// opposite halves of the bank space so a quarter-warp reading rows g, g+1 never conflicts
__device__ __forceinline__ uint32_t page_off(int r, int c) { return r * 512 + ((c ^ ((r & 1) << 2)) << 4); }

// Block id holding tile `tile` of sequence b (a 16-token tile never straddles a block: block % 16 == 0),
// or -1 past the table / out of range (flagged).
__device__ __forceinline__ int tile_block(const AttnParams& P, int b, int tile) {
  const int col = (tile * TILE) / P.block_size;
  if (col >= P.bt_stride) return -1;
  const int blk = P.block_table[b * P.bt_stride + col];
  return (blk >= 0 && blk < P.num_blocks) ? blk : -1;
}

template <int HD, int MAXH>
__global__ void __launch_bounds__(WARPS * 32) paged_attn_split_kernel(const AttnParams P) {
  pdl_trigger();
  pdl_wait();
  static_assert(HD == 128, "head_dim 128");
  constexpr int KP = HD / 32;  // 32-dim slabs: one 16-byte chunk per lane per token row
  extern __shared__ __align__(128) uint8_t smem[];
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int hpk = P.nq / P.nkv;
  const int head0 = kh * hpk;
  const int seqlen = P.seqlens[b];
  const int ntiles = (seqlen + TILE - 1) / TILE;
  const int tile_lo = split * P.tiles_per_split;
  const int tile_hi = min(ntiles, tile_lo + P.tiles_per_split);
  // this warp's tiles: tile_lo + warp + i * WARPS, i < n_w
  const int n_w = tile_hi > tile_lo + warp ? (tile_hi - tile_lo - warp + WARPS - 1) / WARPS : 0;
  const uint32_t ring = static_cast<uint32_t>(__cvta_generic_to_shared(smem)) + warp * STAGES * PAGE_BYTES;

  // Copy page i of this warp into ring slot i % STAGES: lane l moves chunk l of each of the 16 token rows
  // (chunks 0-15 from the key row, 16-31 from the value row); rows past the sequence are zero-filled.
  int blk_next = n_w > 0 ? tile_block(P, b, tile_lo + warp) : -1;
  auto issue = [&](int i) {
    const int tile = tile_lo + warp + i * WARPS;
    const int blk = blk_next;
    if (i + 1 < n_w) blk_next = tile_block(P, b, tile + WARPS);  // one page ahead: hides the table read
    if (blk < 0 && tile * TILE < seqlen) flag_error(P.err, DEVERR_INDEX);
    const int off0 = (tile * TILE) % P.block_size;
    const bf16* base = (lane < 16 ? P.kc : P.vc) + (blk < 0 ? 0 : blk) * P.c_block + kh * P.c_head + (lane & 15) * 8;
    const uint32_t dst = ring + (i % STAGES) * PAGE_BYTES;
#pragma unroll
    for (int r = 0; r < TILE; ++r) {
      const bool valid = blk >= 0 && tile * TILE + r < seqlen;
      cp_async16(dst + page_off(r, lane), base + (off0 + r) * P.c_tok, valid);
    }
  };

  // Query fragments: rows g and g+8 are query heads head0+g, head0+g+8 (zero beyond hpk).
  uint4 qa[KP], qb[KP];
#pragma unroll
  for (int kp = 0; kp < KP; ++kp) {
    qa[kp] = g < hpk ? ld16(P.q + b * P.q_b + (head0 + g) * P.q_h + kp * 32 + 8 * t) : make_uint4(0, 0, 0, 0);
    if constexpr (MAXH > 8)
      qb[kp] = g + 8 < hpk ? ld16(P.q + b * P.q_b + (head0 + g + 8) * P.q_h + kp * 32 + 8 * t) : make_uint4(0, 0, 0, 0);
    else
      qb[kp] = make_uint4(0, 0, 0, 0);
  }

  float o[KP][4][4];
#pragma unroll
  for (int a = 0; a < KP; ++a)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[a][j][e] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < n_w) issue(s);
    cp_async_commit();
  }
  for (int i = 0; i < n_w; ++i) {
    if (i + STAGES - 1 < n_w) issue(i + STAGES - 1);
    cp_async_commit();
    cp_async_wait<STAGES - 1>();
    __syncwarp();
    const uint32_t page = ring + (i % STAGES) * PAGE_BYTES;
    const int tile = tile_lo + warp + i * WARPS;
    uint4 kr[2][KP], vr[2][KP];
#pragma unroll
    for (int kp = 0; kp < KP; ++kp) {
      kr[0][kp] = lds16(page + page_off(g, kp * 4 + t));
      kr[1][kp] = lds16(page + page_off(g + 8, kp * 4 + t));
      vr[0][kp] = lds16(page + page_off(g, 16 + kp * 4 + t));
      vr[1][kp] = lds16(page + page_off(g + 8, 16 + kp * 4 + t));
    }
    __syncwarp();  // the ring slot may be refilled by the next iteration's copy
    // S = Q K^T for the two 8-token halves
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
#pragma unroll
      for (int kp = 0; kp < KP; ++kp) {
        mma_bf16_16816(s[nt], qa[kp].x, qb[kp].x, qa[kp].y, qb[kp].y, kr[nt][kp].x, kr[nt][kp].y);
        mma_bf16_16816(s[nt], qa[kp].z, qb[kp].z, qa[kp].w, qb[kp].w, kr[nt][kp].z, kr[nt][kp].w);
      }
    }
    // scale, mask, online softmax (rows g -> lo, g+8 -> hi)
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = tile * TILE + nt * 8 + 2 * t + (e & 1);
        s[nt][e] = tok < seqlen ? s[nt][e] * P.scale_log2 : -INFINITY;
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
    const float al_lo = exp2f(m_lo - mn_lo), al_hi = exp2f(m_hi - mn_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - mn_lo);
      s[nt][1] = exp2f(s[nt][1] - mn_lo);
      s[nt][2] = exp2f(s[nt][2] - mn_hi);
      s[nt][3] = exp2f(s[nt][3] - mn_hi);
      sum_lo += s[nt][0] + s[nt][1];
      sum_hi += s[nt][2] + s[nt][3];
    }
    l_lo = l_lo * al_lo + sum_lo;
    l_hi = l_hi * al_hi + sum_hi;
#pragma unroll
    for (int a = 0; a < KP; ++a)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[a][j][0] *= al_lo;
        o[a][j][1] *= al_lo;
        o[a][j][2] *= al_hi;
        o[a][j][3] *= al_hi;
      }
    const uint32_t pa0 = pack_bf16x2(s[0][0], s[0][1]), pa1 = pack_bf16x2(s[0][2], s[0][3]);
    const uint32_t pa2 = pack_bf16x2(s[1][0], s[1][1]), pa3 = pack_bf16x2(s[1][2], s[1][3]);
    // O += P V: values transposed 8x8 at a time into B fragments
#pragma unroll
    for (int vp = 0; vp < KP; ++vp) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t b0 = transpose8x8(word(vr[0][vp], j));
        const uint32_t b1 = transpose8x8(word(vr[1][vp], j));
        mma_bf16_16816(o[vp][j], pa0, pa1, pa2, pa3, b0, b1);
      }
    }
  }
  cp_async_wait<0>();

  // row sums live spread over the 4 lanes of a row group
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
  }

  // merge the warps in shared memory (reusing the page rings)
  __syncthreads();
  float (*sm_o)[MAXH][HD] = reinterpret_cast<float (*)[MAXH][HD]>(smem);
  float (*sm_m)[MAXH] = reinterpret_cast<float (*)[MAXH]>(smem + WARPS * MAXH * HD * 4);
  float (*sm_l)[MAXH] = reinterpret_cast<float (*)[MAXH]>(smem + WARPS * MAXH * HD * 4 + WARPS * MAXH * 4);
  if (t == 0) {
    sm_m[warp][g] = m_lo;
    sm_l[warp][g] = l_lo;
    if (MAXH > 8) {
      sm_m[warp][(g + 8) % MAXH] = m_hi;
      sm_l[warp][(g + 8) % MAXH] = l_hi;
    }
  }
#pragma unroll
  for (int vp = 0; vp < KP; ++vp)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int d = vp * 32 + 8 * t + 2 * j;
      sm_o[warp][g][d] = o[vp][j][0];
      sm_o[warp][g][d + 1] = o[vp][j][1];
      if (MAXH > 8) {
        sm_o[warp][(g + 8) % MAXH][d] = o[vp][j][2];
        sm_o[warp][(g + 8) % MAXH][d + 1] = o[vp][j][3];
      }
    }
  __syncthreads();
  for (int idx = threadIdx.x; idx < hpk * HD; idx += blockDim.x) {
    const int r = idx / HD, d = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, sm_m[w][r]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        const float f = exp2f(sm_m[w][r] - M);
        L += sm_l[w][r] * f;
        O += sm_o[w][r][d] * f;
      }
    }
    const int head = head0 + r;
    if (P.splits == 1) {
      P.out[b * P.o_b + head * P.o_h + d] = f2bf(L > 0.f ? O / L : 0.f);
    } else {
      const int64_t slot = (static_cast<int64_t>(b) * P.nq + head) * P.splits + split;
      P.part_o[slot * HD + d] = O;
      if (d == 0) {
        P.part_ml[slot * 2] = M;
        P.part_ml[slot * 2 + 1] = L;
      }
    }
  }
}

constexpr int SPLIT_SMEM = WARPS * STAGES * PAGE_BYTES;  // >= the merge area (4 x 16 x 128 x 4 + 2 x 4 x 16 x 4)
static_assert(SPLIT_SMEM >= WARPS * 16 * 128 * 4 + 2 * WARPS * 16 * 4, "merge area must fit in the page rings");

template <int HD>
__global__ void __launch_bounds__(HD) paged_attn_merge_kernel(const AttnParams P) {
  pdl_trigger();
  pdl_wait();
  const int head = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int64_t base = (static_cast<int64_t>(b) * P.nq + head) * P.splits;
  float M = -INFINITY;
  for (int s = 0; s < P.splits; ++s) M = fmaxf(M, P.part_ml[(base + s) * 2]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < P.splits; ++s) {
      const float f = exp2f(P.part_ml[(base + s) * 2] - M);
      L += P.part_ml[(base + s) * 2 + 1] * f;
      O += P.part_o[(base + s) * HD + d] * f;
    }
  }
  P.out[b * P.o_b + head * P.o_h + d] = f2bf(L > 0.f ? O / L : 0.f);
}

int g_num_sms = 0;
bool g_smem_attr[64] = {};

int sm_count() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" size_t mmp_paged_attn_workspace_size(int batch, int nq, int hd, int splits) {
  if (batch <= 0 || nq <= 0 || hd <= 0 || splits <= 1) return 0;
  return static_cast<size_t>(batch) * nq * splits * (hd + 2) * sizeof(float);
}

// Split count from a waves x tiles-per-warp cost model (2 resident CTAs per SM, STAGES-1 pages of pipeline
// fill per warp, one extra unit for the merge pass when split).
static int choose_splits(int batch, int nkv, int max_tiles) {
  const int slots = 2 * sm_count();
  int best = 1;
  long best_cost = -1;
  for (int s = 1; s <= std::min(64, max_tiles); ++s) {
    const long ctas = static_cast<long>(batch) * nkv * s;
    const long waves = (ctas + slots - 1) / slots;
    const int tps = (max_tiles + s - 1) / s;
    const long cost = waves * ((tps + WARPS - 1) / WARPS + STAGES - 1) + (s > 1 ? 1 : 0);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

extern "C" int mmp_paged_attn_default_splits(int batch, int nkv, int max_seqlen) {
  if (batch <= 0 || nkv <= 0 || max_seqlen < 0) return 1;
  const int max_tiles = std::max(1, (max_seqlen + TILE - 1) / TILE);
  int splits = std::min(choose_splits(batch, nkv, max_tiles), max_tiles);
  const int tps = (max_tiles + splits - 1) / splits;
  return (max_tiles + tps - 1) / tps;
}

extern "C" int mmp_paged_attn_decode(const void* q, int64_t q_b, int64_t q_h,
                                     const void* key_cache, const void* value_cache, int64_t c_block, int64_t c_tok, int64_t c_head,
                                     const int32_t* block_table, int64_t bt_stride, const int32_t* seqlens,
                                     void* out, int64_t o_b, int64_t o_h,
                                     int batch, int nq, int nkv, int hd, int block_size, int num_blocks,
                                     int max_seqlen, float scale, int splits, void* workspace, size_t workspace_bytes,
                                     int* err, void* stream) {
  if (batch == 0) return MMP_OK;
  if (!q || !key_cache || !value_cache || !block_table || !seqlens || !out)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_paged_attn_decode: null pointer");
  if (hd != 128) return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_paged_attn_decode: head_dim %d (only 128)", hd);
  if (batch < 0 || batch > 65535 || nkv <= 0 || nq <= 0 || nq % nkv || nq / nkv > 16 || nkv > 65535 ||
      block_size <= 0 || block_size % TILE || num_blocks <= 0 || max_seqlen < 0)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_paged_attn_decode: bad sizes nq=%d nkv=%d block=%d", nq, nkv, block_size);
  if (!aligned16(q) || !aligned16(key_cache) || !aligned16(value_cache) || q_b % 8 || q_h % 8 || c_block % 8 ||
      c_tok % 8 || c_head % 8)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_paged_attn_decode: q and cache rows must be 16-byte aligned");
  const int max_tiles = std::max(1, (max_seqlen + TILE - 1) / TILE);
  if (splits <= 0) splits = choose_splits(batch, nkv, max_tiles);
  splits = std::min(splits, max_tiles);
  const int tps = (max_tiles + splits - 1) / splits;
  splits = (max_tiles + tps - 1) / tps;
  if (splits > 1 && (!workspace || workspace_bytes < mmp_paged_attn_workspace_size(batch, nq, hd, splits)))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_paged_attn_decode: workspace of %zu bytes needed for %d splits",
                         mmp_paged_attn_workspace_size(batch, nq, hd, splits), splits);
  float* ws = static_cast<float*>(workspace);
  AttnParams P{static_cast<const bf16*>(q), q_b, q_h,
               static_cast<const bf16*>(key_cache), static_cast<const bf16*>(value_cache), c_block, c_tok, c_head,
               block_table, bt_stride, seqlens, static_cast<bf16*>(out), o_b, o_h,
               ws, ws ? ws + static_cast<size_t>(batch) * nq * splits * hd : nullptr,
               batch, nq, nkv, block_size, num_blocks, splits, tps,
               scale * 1.4426950408889634f, err};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(splits, nkv, batch);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !g_smem_attr[dev]) {
    cudaFuncSetAttribute(paged_attn_split_kernel<128, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, SPLIT_SMEM);
    cudaFuncSetAttribute(paged_attn_split_kernel<128, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, SPLIT_SMEM);
    g_smem_attr[dev] = true;
  }
  cudaError_t e = nq / nkv <= 8
                      ? mmp::launch(paged_attn_split_kernel<128, 8>, grid, dim3(WARPS * 32), SPLIT_SMEM, s, nullptr, 0, P)
                      : mmp::launch(paged_attn_split_kernel<128, 16>, grid, dim3(WARPS * 32), SPLIT_SMEM, s, nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_decode: %s", cudaGetErrorString(e));
  int rc = mmp_check_launch("mmp_paged_attn_decode");
  if (rc != MMP_OK || splits == 1) return rc;
  e = mmp::launch(paged_attn_merge_kernel<128>, dim3(nq, batch), dim3(128), 0, s, nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_decode(merge): %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_paged_attn_decode(merge)");
}

// ---------------------------------------------------------------------------------------------------------
// Allocation-free variant of the paged decode attention.
//
// Some callers cannot hand us a workspace: a serving engine that reserved all free HBM for its KV-cache pool
// at start-up (a later cudaMalloc fails or fragments that pool), code that must not call cudaFree (it
// synchronises the whole device), and hosts in other languages that bind only this C ABI and own no device
// allocator. For them the split-K partials live in the fixed array below, which every GPU that loads this
// library holds until the process exits. Its device address is looked up once per device with that device
// current (cudaGetSymbolAddress) on the first call there; make that first call before any stream capture.
// The address is kept until the process exits: after cudaDeviceReset on a device it is stale there.
// All calls share the array, so calls that overlap on the GPU (two streams, two threads) race on it; every
// partial slot the merge reads is rewritten by the same call, so nothing needs clearing between calls.
#include <mutex>

static __device__ __align__(256) float g_attn_noalloc_scratch[MMP_PAGED_ATTN_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {
constexpr int kMaxDevices = 64;
void* g_noalloc_addr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

int noalloc_scratch(void** addr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_paged_attn_decode_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return mmp_set_error(MMP_ERR_CUDA, "mmp_paged_attn_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
  }
  *addr = g_noalloc_addr[dev];
  return MMP_OK;
}
}  // namespace

extern "C" int mmp_paged_attn_decode_noalloc(const void* q, int64_t q_b, int64_t q_h,
                                             const void* key_cache, const void* value_cache, int64_t c_block, int64_t c_tok,
                                             int64_t c_head, const int32_t* block_table, int64_t bt_stride,
                                             const int32_t* seqlens, void* out, int64_t o_b, int64_t o_h,
                                             int batch, int nq, int nkv, int hd, int block_size, int num_blocks,
                                             int max_seqlen, float scale, int splits, int* err, void* stream) {
  if (batch == 0) return MMP_OK;
  if (batch < 0 || nq <= 0 || nkv <= 0 || hd <= 0 || max_seqlen < 0)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_paged_attn_decode_noalloc: bad sizes");
  // the split count the kernel will run with, as mmp_paged_attn_decode normalises it
  const int max_tiles = std::max(1, (max_seqlen + TILE - 1) / TILE);
  int s = splits > 0 ? std::min(splits, max_tiles) : mmp_paged_attn_default_splits(batch, nkv, max_seqlen);
  const int tps = (max_tiles + s - 1) / s;
  s = (max_tiles + tps - 1) / tps;
  const size_t need = mmp_paged_attn_workspace_size(batch, nq, hd, s);
  if (need > MMP_PAGED_ATTN_NOALLOC_SCRATCH_BYTES)
    return mmp_set_error(MMP_ERR_INVALID,
                         "mmp_paged_attn_decode_noalloc: batch %d x %d heads x %d splits needs %zu bytes of scratch, "
                         "more than the %zu bytes this entry point holds; use fewer splits or mmp_paged_attn_decode "
                         "with a workspace", batch, nq, s, need, (size_t)MMP_PAGED_ATTN_NOALLOC_SCRATCH_BYTES);
  void* ws = nullptr;
  if (need > 0) {
    const int rc = noalloc_scratch(&ws);
    if (rc != MMP_OK) return rc;
  }
  return mmp_paged_attn_decode(q, q_b, q_h, key_cache, value_cache, c_block, c_tok, c_head, block_table, bt_stride,
                               seqlens, out, o_b, o_h, batch, nq, nkv, hd, block_size, num_blocks, max_seqlen, scale, s,
                               ws, need > 0 ? (size_t)MMP_PAGED_ATTN_NOALLOC_SCRATCH_BYTES : 0, err, stream);
}
