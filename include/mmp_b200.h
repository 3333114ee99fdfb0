/*
 * libmmp_b200 — C ABI of the B200 (sm_100a) kernels behind the hybrid mixer-layer forward.
 *
 * Every entry point takes raw device pointers, explicit sizes and element strides, and the CUDA stream
 * to launch on; it validates its arguments, launches, and returns a status code (MMP_OK = 0). Nothing
 * here allocates memory or synchronises the host, so every call can be captured in a CUDA graph. The
 * caller owns all buffers. Strides are in elements. bf16 tensors are passed as `void*`.
 *
 * Each function names the reference interface it replaces: the reference harness reaches vLLM's kernels
 * only through harness/kernels.py (anuragdutt/multi_modal_parallelism), whose wrappers are cited by
 * file:line below. A binding generator (ctypes, cffi, cgo) needs only this header.
 */
#ifndef MMP_B200_H_
#define MMP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------------ */
#define MMP_OK 0
#define MMP_ERR_INVALID 1      /* bad shape, stride, dtype, alignment or null pointer */
#define MMP_ERR_CUDA 2         /* a CUDA runtime call or kernel launch failed */
#define MMP_ERR_UNSUPPORTED 3  /* a valid request this build has no kernel for */
#define MMP_ERR_TIMEOUT 4      /* a bounded device-side wait ran out */

/* element types */
#define MMP_F32 0
#define MMP_BF16 1

/* device error-word bits written by kernels that are given an `err` pointer (never a trap) */
#define MMP_DEVERR_INDEX 1
#define MMP_DEVERR_POSITION 2
#define MMP_DEVERR_TIMEOUT 4

/* Library version (major*10000 + minor*100 + patch). */
int mmp_version(void);
/* Programmatic dependent launch (no counterpart in the reference), a bit mask: bit 0 = the tensor-core GEMMs,
 * bit 1 = every other kernel. A kernel so launched starts during the previous kernel's tail and waits for it
 * before touching its outputs; the GEMMs stream their weight operand before that wait. Default 1 (GEMMs only,
 * the faster setting measured on B200). Returns the previous mask. Process-wide; set before capturing graphs. */
int mmp_set_pdl(int enable);
/* Message of the last failing call on this host thread ("" if none). */
const char* mmp_last_error(void);

/* ---- Mamba-2 decode: selective state update -------------------------------------------------------
 * Replaces kernels.ssm_update (harness/kernels.py:137-143), i.e. vLLM selective_state_update with
 * dt_softplus=True, state_batch_indices=idx_in, dst_state_batch_indices=idx_out.
 *   dt' = softplus(dt[b,h] + dt_bias[h]) (or dt + dt_bias when dt_softplus == 0)
 *   s   = state[idx_in[b], h] * exp(dt' A[h]) + dt' x[b,h,:] (outer) B[b,g,:]      -> state[idx_out[b], h]
 *   y   = s C[b,g,:] + D[h] x[b,h,:];  y *= silu(z[b,h,:]) if z != NULL            -> out[b,h,:]
 * with g = h / (nh / ngroups). state: [lines, nh, p, N] (N contiguous), fp32 or bf16. x, z, out: [batch,
 * nh, p] bf16 (p contiguous). dt: [batch, nh] bf16. B, C: [batch, ngroups, N] bf16 (N contiguous).
 * A, D, dt_bias: [nh] fp32 (D, dt_bias may be NULL). idx_in / idx_out: [batch] int32, NULL = identity.
 * A row whose idx_in equals pad_slot is skipped (its state lines are not touched; its output row is 0).
 * Supported: N in {64, 128, 256}; all rows 16-byte aligned.
 */
int mmp_ssu_decode(void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                   const void* x, int64_t x_b, int64_t x_h,
                   const void* dt, int64_t dt_b, int64_t dt_h,
                   const float* A, const float* D, const float* dt_bias,
                   const void* B, int64_t B_b, int64_t B_g,
                   const void* C, int64_t C_b, int64_t C_g,
                   const void* z, int64_t z_b, int64_t z_h,
                   const int32_t* idx_in, const int32_t* idx_out, int pad_slot,
                   void* out, int64_t o_b, int64_t o_h,
                   int batch, int nh, int p, int N, int ngroups, int lines, int dt_softplus,
                   int* err, void* stream);

/* ---- Mamba-2 decode: causal depthwise conv update -------------------------------------------------
 * Replaces kernels.conv_update (harness/kernels.py:131-134), i.e. vLLM causal_conv1d_update with
 * activation "silu" and conv_state_indices. For each row b with line = idx[b]:
 *   window = [state[line, 0..W-2, c], x[b, c]]; out[b,c] = act(sum_k w[c,k] window[k] + bias[c])
 *   state[line, k, c] = window[k+1]
 * x, out: [batch, rows] bf16 (out may alias x). state: element (line, k, c) at line*s_line + k*s_k + c*s_c
 * (bf16). w: [rows, W] bf16 contiguous; bias: [rows] bf16 or NULL. Rows with idx == pad_slot are
 * skipped (output row 0). W <= 8.
 */
int mmp_conv1d_update(const void* x, int64_t x_b, void* out, int64_t o_b,
                      void* state, int64_t s_line, int64_t s_k, int64_t s_c,
                      const void* w, const void* bias, const int32_t* idx, int pad_slot,
                      int batch, int rows, int W, int lines, int silu, int* err, void* stream);

/* ---- RMSNorm (+ residual) -------------------------------------------------------------------------
 * Replaces kernels.rms_norm (harness/kernels.py:26-28). out = x * rsqrt(mean(x^2) + eps) * w over rows
 * of length `hidden`. With `residual` != NULL the normalised value is x + residual, and that sum is also
 * written to `sum_out` (may alias x or residual) — the layer's `h1 = h + mix` fused with the next norm.
 * All bf16, row strides in elements, rows 16-byte aligned, hidden % 8 == 0.
 */
int mmp_rmsnorm(const void* x, int64_t x_b, const void* residual, int64_t r_b, void* sum_out, int64_t s_b,
                const void* w, void* out, int64_t o_b, int rows, int hidden, float eps, void* stream);

/* ---- Mamba-2 gated RMSNorm (norm after the gate) --------------------------------------------------
 * Replaces kernels.gated_rmsnorm (harness/kernels.py:40-52) with its local path (group == None) and
 * both halves of its tensor-parallel path:
 *   g = y * silu(z);  out = w * g * rsqrt(sumsq(g over the group) / count + eps)
 * mode 0 (local): groups of `group_size` columns, reduced inside the kernel.
 * mode 1 (partial): write each row's per-group sum of squares to sumsq [rows, D/group_size] fp32 and
 *   nothing else — the caller reduces it across the ranks of the norm group.
 * mode 2 (apply): use the reduced sums in sumsq with `count` elements per group.
 * mode 3 (deferred): write the partial sums as mode 1 and out = w * g unnormalised; once the sums are reduced,
 *   mmp_scale_rows applies the normalisation to any product linear in the rows of out (the out-projection), so
 *   the reduction can run while that product is computed.
 * y, z, out: [rows, D] bf16 with row strides; w: [D] bf16.
 */
int mmp_gated_rmsnorm(const void* y, int64_t y_b, const void* z, int64_t z_b, const void* w,
                      void* out, int64_t o_b, float* sumsq, int rows, int D, int group_size,
                      int mode, float count, float eps, void* stream);

/* x[r, :] *= rsqrt(sumsq[r] / count + eps), in place: the normalisation deferred by mmp_gated_rmsnorm mode 3, applied
 * to the rows of a product of the unnormalised values (one group per row: sumsq [rows] fp32, reduced over the norm
 * group's ranks; count = the group's full width). x: [rows, cols] bf16, row stride ld, cols % 8 == 0, 16-byte
 * aligned rows. No counterpart in the reference: its tensor-parallel norm always reduces before the projection. */
int mmp_scale_rows(void* x, int64_t ld, const float* sumsq, int rows, int cols, float count, float eps, void* stream);

/* ---- RoPE + key multiplier + paged KV write --------------------------------------------------------
 * Replaces kernels.apply_rope and kernels.write_kv (harness/kernels.py:56-66,112-115) and the layer's
 * `k * key_mult` (harness/layer.py:35), fused into one pass over the QKV projection output.
 * q: [batch, nq*hd], k / v: [batch, nkv*hd] bf16 (row strides q_b, k_b, v_b; they may be column slices
 * of one [q | k | v] row). With positions != NULL, q and k*key_mult are rotated NeoX-style (rotate
 * halves) at positions[b]; cos/sin come from `cos_sin` ([max_pos, hd] fp32 = cat(cos, sin)) when
 * non-NULL, else from `inv_freq` ([hd/2] fp32). positions == NULL: no rotation, no multiplier.
 * Rotated q goes to q_out (may alias q); rotated k to k_out when non-NULL (may alias k). When key_cache is
 * non-NULL, k and v are written to the paged caches at slot_mapping[b] (skipped when < 0); caches are
 * [num_blocks, block, nkv, hd] views with element strides (c_block, c_tok, c_head).
 */
int mmp_rope_kv_write(const void* q, int64_t q_b, const void* k, int64_t k_b, const void* v, int64_t v_b,
                      int nq, int nkv, int hd, const int64_t* positions, const float* cos_sin, int max_pos,
                      const float* inv_freq, float key_mult,
                      void* q_out, int64_t qo_b, void* k_out, int64_t ko_b,
                      void* key_cache, void* value_cache, int64_t c_block, int64_t c_tok, int64_t c_head,
                      int block_size, int num_blocks, const int64_t* slot_mapping,
                      int batch, int* err, void* stream);

/* ---- SwiGLU activation ----------------------------------------------------------------------------
 * Replaces kernels.silu_and_mul (harness/kernels.py:31-37) and the MLP's `F.silu(g * gm) * u`
 * (harness/layer.py:135): out[r, c] = silu(gate_scale * gate[r, c]) * up[r, c], bf16, row strides in
 * elements (cols % 8 == 0, 16-byte aligned rows).
 */
int mmp_silu_mul(const void* gate, int64_t g_b, const void* up, int64_t u_b, void* out, int64_t o_b,
                 int rows, int cols, float gate_scale, void* stream);

/* ---- paged GQA decode attention -------------------------------------------------------------------
 * Replaces kernels.attn_decode (harness/kernels.py:118-127), i.e. FlashAttention-2 varlen with
 * max_seqlen_q = 1, a block table and seqused_k. One query token per sequence; query head i reads KV
 * head i / (nq / nkv). q: [batch, nq, hd] bf16; caches as in mmp_rope_kv_write; block_table:
 * [batch, bt_stride] int32; seqlens: [batch] int32 keys per sequence; out: [batch, nq, hd] bf16.
 * The key range of a sequence is split over `splits` CTAs whose partial results go to `workspace`
 * (size from mmp_paged_attn_workspace_size) and are merged by a second kernel. splits <= 0 picks a
 * split count for this GPU. Supported: hd == 128, block % 16 == 0, nq / nkv <= 16.
 */
size_t mmp_paged_attn_workspace_size(int batch, int nq, int hd, int splits);
/* The split count mmp_paged_attn_decode picks for splits <= 0 (for sizing the workspace once). */
int mmp_paged_attn_default_splits(int batch, int nkv, int max_seqlen);
int mmp_paged_attn_decode(const void* q, int64_t q_b, int64_t q_h,
                          const void* key_cache, const void* value_cache, int64_t c_block, int64_t c_tok, int64_t c_head,
                          const int32_t* block_table, int64_t bt_stride, const int32_t* seqlens,
                          void* out, int64_t o_b, int64_t o_h,
                          int batch, int nq, int nkv, int hd, int block_size, int num_blocks,
                          int max_seqlen, float scale, int splits, void* workspace, size_t workspace_bytes,
                          int* err, void* stream);

/* ---- paged GQA decode attention without a caller workspace --------------------------------------------
 * No counterpart in the reference. For callers that cannot allocate device memory — an engine that has
 * already reserved the free HBM for its own pools, code that must not call cudaFree (it synchronises the
 * device), or a foreign-language host that binds only this ABI — this variant of mmp_paged_attn_decode
 * keeps its split-K partials in a fixed scratch array of MMP_PAGED_ATTN_NOALLOC_SCRATCH_BYTES (8 MiB) inside
 * the library, held by every GPU that loads it until the process exits. Same arguments and results as
 * mmp_paged_attn_decode without the workspace; returns MMP_ERR_INVALID when batch x nq x splits x
 * (hd + 2) x 4 bytes exceeds the array. The first call on a device looks up the array's address there:
 * make it before any stream capture. The address is kept for the life of the process, so do not call
 * this entry point on a device after cudaDeviceReset there. Calls share the array: calls that overlap on
 * the GPU race.
 */
#define MMP_PAGED_ATTN_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)
int mmp_paged_attn_decode_noalloc(const void* q, int64_t q_b, int64_t q_h,
                                  const void* key_cache, const void* value_cache, int64_t c_block, int64_t c_tok,
                                  int64_t c_head, const int32_t* block_table, int64_t bt_stride,
                                  const int32_t* seqlens, void* out, int64_t o_b, int64_t o_h,
                                  int batch, int nq, int nkv, int hd, int block_size, int num_blocks,
                                  int max_seqlen, float scale, int splits, int* err, void* stream);

/* ---- bf16 GEMM with fused epilogue ----------------------------------------------------------------
 * Replaces kernels.gemm / gemm_T (harness/kernels.py:147-154) together with the scaling the layer
 * applies to their results (harness/layer.py:35,80,105): out[m,n] = alpha * colscale[n] * sum_k
 * a[m,k] w[n,k] + addend[m,n]. a: [M, K] bf16 (row stride lda); w: [N, K] bf16 (row stride ldw);
 * colscale: [N] fp32 or NULL; addend: [M, N] bf16 (row stride ldd) or NULL; out: [M, N] bf16 (row
 * stride ldo, may alias addend). K % 8 == 0, strides % 8 == 0, 16-byte aligned bases.
 */
int mmp_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int64_t ldo,
                  int M, int N, int K, float alpha, const float* colscale, const void* addend, int64_t ldd,
                  void* stream);

/* ---- bf16 GEMM on the tensor cores (tcgen05 / TMEM / TMA) ---------------------------------------------
 * Same contract as mmp_gemm_bf16 (harness/kernels.py:147-154 plus the layer's scalings), computed with
 * 128-row UMMA tiles fed by TMA: M <= 256 runs weight-streaming (the weight rows are the MMA's M side,
 * split-K over a thread-block cluster when the tiles cannot fill the GPU); larger M runs 128 x 256 tiles.
 * err: optional device error word (MMP_DEVERR_TIMEOUT if a pipeline wait ran out).
 */
int mmp_gemm_bf16_tc(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int64_t ldo,
                     int M, int N, int K, float alpha, const float* colscale, const void* addend, int64_t ldd,
                     int* err, void* stream);

/* Split-K count of the decode (M <= 256) weight-streaming GEMMs: 0 (default) picks it from the tile count (enough
 * CTAs to fill the GPU, at most 8, as a thread-block cluster); n > 0 uses min(n, 8) (1: no split). A tuning and
 * measurement switch for the same operation (results differ only by the order of the fp32 partial sums);
 * process-wide; returns the previous setting. No counterpart in the reference (cuBLAS picks its own split). */
int mmp_set_gemm_decode_split(int split);
/* Ring depth of the decode GEMMs with at most 64 activation rows: 4 stages (two CTAs per SM) or 8 (one CTA per SM,
 * twice the weight bytes in flight per CTA); other values select 4. A tuning switch like the one above; returns
 * the previous setting. No counterpart in the reference. */
int mmp_set_gemm_decode_stages(int stages);

/* ---- bf16 GEMM over two K segments with their own scales ---------------------------------------------
 * Replaces the reference layer's two output projections and their sum (harness/layer.py:51-53,103-105,
 * 213-219: o_proj * attn_out + out_proj * ssm_out) when one rank holds both branches: with the two
 * activations side by side in `a` and the two weights side by side in `w`,
 *   out = alpha * a[:, :k_seg] w[:, :k_seg]^T + alpha2 * a[:, k_seg:] w[:, k_seg:]^T, then colscale, addend.
 * k_seg is a multiple of 64 (k_seg >= K: one segment). Otherwise as mmp_gemm_bf16_tc.
 */
int mmp_gemm_bf16_seg(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int64_t ldo,
                      int M, int N, int K, float alpha, int k_seg, float alpha2, const float* colscale,
                      const void* addend, int64_t ldd, int* err, void* stream);

/* ---- prefill: causal depthwise conv over variable-length sequences --------------------------------------
 * The prefill counterpart of mmp_conv1d_update (vLLM causal_conv1d_fn in the stack the reference measures;
 * the reference harness itself only decodes). Tokens [cu_seqlens[i], cu_seqlens[i+1]) form sequence i:
 * out[t, c] = act(bias[c] + sum_k w[c, k] x[t - W + 1 + k, c]), inputs before the sequence's first token taken
 * from state line state_idx[i] (oldest first) when has_init[i] != 0, else zero; then the line receives the
 * sequence's last W-1 inputs. x, out: [ntok, rows] bf16 (out must not alias x); state element (line, k, c) at
 * line*s_line + k*s_k + c. W == 4, rows % 8 == 0, 16-byte aligned rows. has_init may be NULL (no initial state).
 */
int mmp_conv1d_prefill(const void* x, int64_t x_t, void* out, int64_t o_t, void* state, int64_t s_line, int64_t s_k,
                       const void* w, const void* bias, const int32_t* cu_seqlens, const int32_t* state_idx,
                       const int32_t* has_init, int nseq, int ntok, int rows, int W, int lines, int silu,
                       int* err, void* stream);

/* ---- prefill: Mamba-2 chunked SSD scan over variable-length sequences ---------------------------------
 * The prefill counterpart of mmp_ssu_decode (vLLM mamba_chunk_scan_combined_varlen in the stack the reference
 * measures). For each sequence i and head h, runs s_t = exp(dt'_t A) s_{t-1} + dt'_t x_t B_t^T,
 * y_t = s_t C_t + D x_t over its tokens (dt' = softplus(dt + dt_bias)), starting from state line state_idx[i]
 * when has_init[i] != 0 (else zero) and writing the final state back to that line; evaluated chunk-wise (64
 * tokens) on the tensor cores (tcgen05 with TMEM-resident state for p = 128 with N in {128, 256}, and for p = 64
 * with N = 128 when each B/C group has an even number of heads, two heads per CTA; mma.sync otherwise). x, out:
 * [ntok, nh, p] bf16 (ntok = cu_seqlens[nseq], the packed rows); dt: [ntok, nh] bf16; B, C: [ntok, ngroups, N]
 * bf16; state as mmp_ssu_decode. N in {64, 128, 256}, p % 8 == 0, 16-byte aligned rows.
 */
int mmp_ssd_prefill(const void* x, int64_t x_t, int64_t x_h, const void* dt, int64_t dt_t, int64_t dt_h,
                    const float* A, const float* D, const float* dt_bias,
                    const void* B, int64_t B_t, int64_t B_g, const void* C, int64_t C_t, int64_t C_g,
                    void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                    const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init,
                    void* out, int64_t o_t, int64_t o_h,
                    int nseq, int ntok, int nh, int p, int N, int ngroups, int lines, int* err, void* stream);
/* Selects the kernel behind mmp_ssd_prefill: 1 (default) the tcgen05 kernel where it applies, 0 the mma.sync kernel
 * always (no counterpart in the reference; for comparisons). Process-wide; returns the previous setting. */
int mmp_set_ssd_prefill_tc(int enable);

/* ---- prefill: the chunked SSD scan with balanced walks ---------------------------------------------------
 * Same result as mmp_ssd_prefill (up to rounding) for head dim 128. The host cuts each sequence at 64-token chunk
 * boundaries into segments (vcu: [nvirt + 1] packed-row offsets; sequence i owns segments [seg0[i], seg0[i + 1]));
 * the scan runs them as independent sequences with their states in `scratch` ([scratch_lines][nh][128][N] fp32,
 * contiguous; vline[v] = v, vinit[v] = has_init of a sequence's first segment, else 0), so more, shorter walks
 * fill the SMs; then one kernel per (head, sequence) chains the segment states, adds exp(cum_t) S_in C_t to the
 * later segments' outputs and writes the final state to line state_idx[i]. A sequence that continues
 * (has_init[i]) first has its line copied to its first segment's scratch line. Other arguments as
 * mmp_ssd_prefill (cu_seqlens of the sequences is implied by vcu and seg0).
 */
int mmp_ssd_prefill_seg(const void* x, int64_t x_t, int64_t x_h, const void* dt, int64_t dt_t, int64_t dt_h,
                        const float* A, const float* D, const float* dt_bias,
                        const void* B, int64_t B_t, int64_t B_g, const void* C, int64_t C_t, int64_t C_g,
                        void* state, int state_dtype, int64_t s_line, int64_t s_head, int64_t s_p,
                        const int32_t* state_idx, const int32_t* has_init, void* out, int64_t o_t, int64_t o_h,
                        const int32_t* vcu, const int32_t* vline, const int32_t* vinit, const int32_t* seg0,
                        float* scratch, int scratch_lines, int nvirt, int nseq, int ntok, int nh, int p, int N,
                        int ngroups, int lines, int* err, void* stream);

/* ---- prefill: causal GQA attention over the paged KV cache ----------------------------------------------
 * The prefill counterpart of mmp_paged_attn_decode (FlashAttention-2 varlen, causal). Query token j of
 * sequence i (rows [cu_q[i], cu_q[i+1]) of q) sits at position ctx_start[i] + j and attends to cache positions
 * 0 .. ctx_start[i] + j of that sequence, whose keys/values (the new tokens' included) are already in the
 * cache. q: [ntok, nq, hd]; out: [ntok, nq, hd] bf16; caches and block_table as mmp_paged_attn_decode.
 * hd == 128; max_q_len bounds cu_q[i+1] - cu_q[i].
 */
int mmp_paged_attn_prefill(const void* q, int64_t q_t, int64_t q_h,
                           const void* key_cache, const void* value_cache, int64_t c_block, int64_t c_tok,
                           int64_t c_head, const int32_t* block_table, int64_t bt_stride,
                           const int32_t* cu_q, const int32_t* ctx_start, void* out, int64_t o_t, int64_t o_h,
                           int nseq, int max_q_len, int nq, int nkv, int hd, int block_size, int num_blocks,
                           float scale, int* err, void* stream);

/* Selects the kernel behind mmp_paged_attn_prefill: 1 (default) the tcgen05/TMEM kernel (one CTA per pair of query
 * heads sharing a key/value head, S, P and O in tensor memory, paged K/V gathered by TMA, lazy softmax rescaling)
 * for requests it fits (head dim 128, page of 8-128 tokens, a power of two; 16-byte aligned output rows), the
 * mma.sync kernel otherwise; 0 the mma.sync kernel always. Process-wide; returns the previous setting. */
int mmp_set_attn_prefill_tc(int enable);

/* ---- elementwise add (residual joins after a collective) -------------------------------------------
 * Replaces the layer's bf16 `a + b (+ c)` residual sums (harness/layer.py:217-219,225-227):
 * out = a + b (+ c when c != NULL), computed in fp32, rounded once to bf16. [rows, cols] with row strides
 * (cols % 8 == 0, 16-byte aligned rows); out may alias an input.
 */
int mmp_add(const void* a, int64_t a_b, const void* b, int64_t b_b, const void* c, int64_t c_b,
            void* out, int64_t o_b, int rows, int cols, void* stream);

/* ---- Gated DeltaNet linear attention (the config's gated delta-rule layers) ----------------------------
 * The reference has no kernel for these layers: configs/qwen35_35b_a3b.yaml:1-22 describes them and
 * harness/synth.py:114-138 models their bytes. Per value head j (key head j / (nv / nk)), with q, k the
 * post-conv rows L2-normalised in fp32 (q also scaled by dk^-1/2), g = -exp(A_log[j]) softplus(a + dt_bias[j])
 * (A_log / dt_bias NULL: factor 1 / bias 0), beta = sigmoid(b):
 *   S <- exp(g) S (I - beta k k^T) + beta v k^T,   o = S q,
 * S the [dv, dk] fp32 state of the line. Output: rmsnorm(o) * norm_w * silu(z) over the head's dv values
 * (norm_w NULL: o itself; z NULL: no gate; eps for the norm). dk == dv == 128.
 *
 * Decode: one token per row. q/k [batch, nk, dk], v/z/out [batch, nv, dv], a/b [batch, nv] (raw projections,
 * heads contiguous), state [lines, nv, dv, dk] fp32, idx[row] its line (NULL: the row index; pad_slot: the
 * row's output is zero and no state is touched; out-of-range lines set MMP_DEVERR_INDEX in *err).
 */
int mmp_gdn_decode(float* state, int64_t s_line, int64_t s_head, int64_t s_row,
                   const void* q, int64_t q_b, int64_t q_h, const void* k, int64_t k_b, int64_t k_h,
                   const void* v, int64_t v_b, int64_t v_h, const void* a, int64_t a_b,
                   const void* b, int64_t b_b, const float* A_log, const float* dt_bias,
                   const void* z, int64_t z_b, int64_t z_h, const void* norm_w, float eps,
                   const int32_t* idx, int pad_slot, void* out, int64_t o_b, int64_t o_h,
                   int batch, int nk, int nv, int dk, int dv, int lines, int* err, void* stream);

/* Chunked prefill (64-token chunks) of variable-length sequences: tokens [cu_seqlens[i], cu_seqlens[i+1]) of
 * q/k [ntok, nk, dk], v/z/out [ntok, nv, dv], a/b [ntok, nv]; sequence i starts from state line state_idx[i]
 * when has_init[i] (has_init NULL: from zeros) and leaves its final state there. Rows 16-byte aligned. */
int mmp_gdn_prefill(const void* q, int64_t q_t, int64_t q_h, const void* k, int64_t k_t, int64_t k_h,
                    const void* v, int64_t v_t, int64_t v_h, const void* a, int64_t a_t,
                    const void* b, int64_t b_t, const float* A_log, const float* dt_bias,
                    const void* z, int64_t z_t, int64_t z_h, const void* norm_w, float eps,
                    float* state, int64_t s_line, int64_t s_head, int64_t s_row,
                    const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init,
                    void* out, int64_t o_t, int64_t o_h,
                    int nseq, int ntok, int nk, int nv, int dk, int dv, int lines, int* err, void* stream);

/* The same chunked prefill on the tensor cores, in two passes: every chunk of every sequence at once (the chunk's
 * [K; Q] K^T on tcgen05, the inverse of its unit lower-triangular matrix T in fp32, T and the masked Q K^T
 * written to `workspace` as bf16), then one walk per (value head, sequence) with the state in tensor memory.
 * Arguments as mmp_gdn_prefill; q/k/v/z/out additionally need 16-byte aligned rows and head strides. workspace:
 * 16-byte aligned, at least mmp_gdn_prefill_workspace_size(ntok, nv) bytes; its contents are scratch.
 * Same results as mmp_gdn_prefill within bf16 rounding (the chunk algebra is regrouped, not changed). */
size_t mmp_gdn_prefill_workspace_size(int ntok, int nv);
int mmp_gdn_prefill_tc(const void* q, int64_t q_t, int64_t q_h, const void* k, int64_t k_t, int64_t k_h,
                       const void* v, int64_t v_t, int64_t v_h, const void* a, int64_t a_t,
                       const void* b, int64_t b_t, const float* A_log, const float* dt_bias,
                       const void* z, int64_t z_t, int64_t z_h, const void* norm_w, float eps,
                       float* state, int64_t s_line, int64_t s_head, int64_t s_row,
                       const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init,
                       void* out, int64_t o_t, int64_t o_h,
                       int nseq, int ntok, int nk, int nv, int dk, int dv, int lines,
                       void* workspace, size_t workspace_bytes, int* err, void* stream);

/* ---- peer-memory all-reduce fused with the residual add and RMSNorm (decode-sized messages) ------------
 * Replaces the NCCL all-reduce of the layer's partial sums (`ParallelHybridLayer._ar`, harness/layer.py:175-181)
 * and the residual / pre-MLP norm after it (harness/layer.py:217-227) on ranks of one node.
 *
 * Buffers: every rank allocates mmp_ar_buffer_bytes(world, rows_max, H) bytes of zeroed device memory, exports it
 * with mmp_ipc_export (MMP_IPC_BLOB_BYTES opaque bytes), exchanges the blobs with the other ranks (any host
 * channel) and maps theirs with mmp_ipc_import; `bufs` is a device array of the world's buffer addresses in
 * this process (own at index rank). mmp_ipc_release unmaps an imported buffer.
 *
 * mmp_ar_join: sum_out = resid + bf16(sum over ranks of part), and, with norm_w, norm_out = rmsnorm(sum_out) *
 * norm_w. part / resid / sum_out / norm_out are [rows, H] bf16 with row strides (16-byte aligned rows; sum_out
 * may alias resid; resid may be NULL). Every rank must make the same sequence of calls on its buffer (a device
 * epoch counts them); results are bit-identical on every rank. A wait that runs out sets MMP_DEVERR_TIMEOUT in
 * *err. world <= 8; rows <= rows_max. pushed = 1: the partial was produced by mmp_gemm_bf16_push on every rank
 * (already in the buffers; `part` is ignored), so this call only waits, sums and normalises.
 *
 * mmp_gemm_bf16_push: the decode GEMM (M <= 256 rows; arguments as mmp_gemm_bf16_seg, no addend) whose output
 * tiles go straight into slot `rank` of every rank's all-reduce buffer instead of a local array, each CTA adding
 * the number of elements it wrote to its counter on every rank: the transfer over NVLink overlaps the GEMM. The
 * mmp_ar_join(pushed = 1) that follows on the same buffer completes the all-reduce. N must equal the buffer's H. */
#define MMP_IPC_BLOB_BYTES 72
size_t mmp_ar_buffer_bytes(int world, int rows_max, int H);
int mmp_ipc_export(const void* ptr, void* blob);
int mmp_ipc_import(const void* blob, void** ptr_out);
int mmp_ipc_release(void* ptr);
int mmp_ar_join(const uint64_t* bufs, int rank, int world, int rows_max, int pushed,
                const void* part, int64_t p_b, const void* resid, int64_t r_b,
                void* sum_out, int64_t s_b, const void* norm_w, float eps, void* norm_out, int64_t n_b,
                int rows, int H, int* err, void* stream);
int mmp_gemm_bf16_push(const void* a, int64_t lda, const void* w, int64_t ldw, int M, int N, int K, float alpha,
                       int k_seg, float alpha2, const float* colscale, const uint64_t* bufs, int rank, int world,
                       int rows_max, int* err, void* stream);

/* Gated RMSNorm whose row statistic spans a norm group's ranks (replaces the tensor-parallel path of
 * kernels.gated_rmsnorm, harness/kernels.py:47-52: local sums of squares, an all-reduce of [rows, 1] over the
 * norm group, the normalisation) in one kernel over peer memory: out = w * g * rsqrt(sum over ranks of
 * sum(g^2) / (world * D) + eps), g = y * silu(z), each rank holding D columns of every row. Buffers as above with
 * mmp_gn_buffer_bytes(world, rows_max) bytes per rank (zeroed, shared with mmp_ipc_export / mmp_ipc_import).
 * y, z, out: [rows, D] bf16 with row strides; w: [D] bf16. Every rank of the group makes the same calls. */
size_t mmp_gn_buffer_bytes(int world, int rows_max);
int mmp_gated_rmsnorm_p2p(const uint64_t* bufs, int rank, int world, int rows_max,
                          const void* y, int64_t y_b, const void* z, int64_t z_b, const void* w,
                          void* out, int64_t o_b, int rows, int D, float eps, int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MMP_B200_H_ */
