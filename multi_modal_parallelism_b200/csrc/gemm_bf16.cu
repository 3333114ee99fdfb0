// mmp_gemm_bf16: the layer's bf16 projection GEMM with fused epilogue (replaces F.linear / @ and the scalings
// the reference layer applies to their results, harness/kernels.py:147-154 and harness/layer.py:35,80,105).
// It runs the tcgen05 tensor-core kernel of gemm_tc.cu.
#include "mmp_common.cuh"

extern "C" int mmp_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int64_t ldo,
                             int M, int N, int K, float alpha, const float* colscale, const void* addend, int64_t ldd,
                             void* stream) {
  return mmp_gemm_bf16_tc(a, lda, w, ldw, out, ldo, M, N, K, alpha, colscale, addend, ldd, nullptr, stream);
}
