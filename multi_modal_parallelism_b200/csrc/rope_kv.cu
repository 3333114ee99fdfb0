// RoPE (NeoX, rotate halves) on q and k, the key multiplier, and the paged KV-cache write in one pass
// (replaces vLLM rotary_embedding + reshape_and_cache_flash and the layer's `k * key_mult`,
// harness/kernels.py:56-66,112-115 and harness/layer.py:35 of the reference).
//
// One warp per (token, head) over the nq + nkv + nkv heads of a row: lane l owns the rotation pairs
// (i, i + hd/2) for i in [l*hd/64, (l+1)*hd/64). Angles are pos * inv_freq in fp32 with sincosf, or come
// from a cos/sin table when the caller passes one; positions == NULL means no rotation (plain cache write).
#include "mmp_common.cuh"

namespace mmp {
namespace {

struct RopeParams {
  const bf16* q; int64_t q_b;
  const bf16* k; int64_t k_b;
  const bf16* v; int64_t v_b;
  int nq, nkv;
  const int64_t* positions;
  const float* cos_sin; int max_pos;
  const float* inv_freq;
  float key_mult;
  bf16* q_out; int64_t qo_b;
  bf16* k_out; int64_t ko_b;
  bf16* kc; bf16* vc; int64_t c_block, c_tok, c_head;
  int block_size, num_blocks;
  const int64_t* slot_mapping;
  int* err;
};

template <int HD>
__global__ void __launch_bounds__(128) rope_kv_kernel(const RopeParams P) {
  pdl_trigger();
  pdl_wait();
  constexpr int PER = HD / 64;  // rotation pairs per lane
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.x * 4 + warp;
  const int b = blockIdx.y;
  const bool has_cache = P.kc != nullptr;
  const int nheads = P.nq + P.nkv + (has_cache ? P.nkv : 0);
  if (head >= nheads) return;
  const bool is_q = head < P.nq;
  const bool is_v = head >= P.nq + P.nkv;
  const int kvh = is_q ? 0 : (is_v ? head - P.nq - P.nkv : head - P.nq);
  const bf16* src = is_q ? P.q + b * P.q_b + head * HD : is_v ? P.v + b * P.v_b + kvh * HD : P.k + b * P.k_b + kvh * HD;
  const int i0 = lane * PER;
  float lo[PER], hi[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    lo[j] = bf2f(src[i0 + j]);
    hi[j] = bf2f(src[i0 + j + HD / 2]);
  }
  if (!is_v && P.positions) {
    const int64_t pos = P.positions[b];
    const float mult = is_q ? 1.f : P.key_mult;
    if (P.cos_sin && (pos < 0 || pos >= P.max_pos)) {
      flag_error(P.err, DEVERR_POSITION);
      return;
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      float c, s;
      if (P.cos_sin) {
        c = P.cos_sin[pos * HD + i0 + j];
        s = P.cos_sin[pos * HD + HD / 2 + i0 + j];
      } else {
        sincosf(static_cast<float>(pos) * P.inv_freq[i0 + j], &s, &c);
      }
      const float a = lo[j] * mult, bb = hi[j] * mult;
      lo[j] = a * c - bb * s;
      hi[j] = bb * c + a * s;
    }
  }
  bf16* dst = nullptr;
  if (is_q) {
    dst = P.q_out + b * P.qo_b + head * HD;
  } else if (!is_v && P.k_out) {
    bf16* kd = P.k_out + b * P.ko_b + kvh * HD;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      kd[i0 + j] = f2bf(lo[j]);
      kd[i0 + j + HD / 2] = f2bf(hi[j]);
    }
  }
  if (!is_q && has_cache) {
    const int64_t slot = P.slot_mapping[b];
    if (slot < 0) return;  // padding row: nothing cached
    const int64_t blk = slot / P.block_size, tok = slot % P.block_size;
    if (blk >= P.num_blocks) {
      flag_error(P.err, DEVERR_INDEX);
      return;
    }
    dst = (is_v ? P.vc : P.kc) + blk * P.c_block + tok * P.c_tok + kvh * P.c_head;
  }
  if (dst) {
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      dst[i0 + j] = f2bf(lo[j]);
      dst[i0 + j + HD / 2] = f2bf(hi[j]);
    }
  }
}

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" int mmp_rope_kv_write(const void* q, int64_t q_b, const void* k, int64_t k_b, const void* v, int64_t v_b,
                                 int nq, int nkv, int hd, const int64_t* positions, const float* cos_sin, int max_pos,
                                 const float* inv_freq, float key_mult,
                                 void* q_out, int64_t qo_b, void* k_out, int64_t ko_b,
                                 void* key_cache, void* value_cache, int64_t c_block, int64_t c_tok, int64_t c_head,
                                 int block_size, int num_blocks, const int64_t* slot_mapping,
                                 int batch, int* err, void* stream) {
  if (batch == 0) return MMP_OK;
  const bool cache = key_cache != nullptr;
  if ((nq > 0 && (!q || !q_out)) || (nkv > 0 && !k) || (cache && (!value_cache || !v || !slot_mapping)) ||
      (positions && !cos_sin && !inv_freq))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_rope_kv_write: null pointer");
  if (batch < 0 || batch > 65535 || nq < 0 || nkv < 0 || nq + nkv == 0 || (cache && (block_size <= 0 || num_blocks <= 0)))
    return mmp_set_error(MMP_ERR_INVALID, "mmp_rope_kv_write: bad sizes");
  RopeParams P{static_cast<const bf16*>(q), q_b, static_cast<const bf16*>(k), k_b, static_cast<const bf16*>(v), v_b,
               nq, nkv, positions, cos_sin, max_pos, inv_freq, key_mult,
               static_cast<bf16*>(q_out), qo_b, static_cast<bf16*>(k_out), ko_b,
               static_cast<bf16*>(key_cache), static_cast<bf16*>(value_cache), c_block, c_tok, c_head,
               block_size, num_blocks, slot_mapping, err};
  dim3 grid((nq + 2 * nkv + 3) / 4, batch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (hd) {
    case 64: { cudaError_t e = mmp::launch(rope_kv_kernel<64>, grid, dim3(128), 0, s, nullptr, 0, P); if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_rope_kv_write: %s", cudaGetErrorString(e)); break; }
    case 128: { cudaError_t e = mmp::launch(rope_kv_kernel<128>, grid, dim3(128), 0, s, nullptr, 0, P); if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_rope_kv_write: %s", cudaGetErrorString(e)); break; }
    case 256: { cudaError_t e = mmp::launch(rope_kv_kernel<256>, grid, dim3(128), 0, s, nullptr, 0, P); if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_rope_kv_write: %s", cudaGetErrorString(e)); break; }
    default: return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_rope_kv_write: head_dim %d not in {64, 128, 256}", hd);
  }
  return mmp_check_launch("mmp_rope_kv_write");
}
