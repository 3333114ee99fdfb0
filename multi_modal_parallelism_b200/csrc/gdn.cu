// Gated DeltaNet (gated delta rule) linear attention: decode (one token per sequence) and chunked prefill over
// variable-length sequences, each with the per-head gated RMSNorm of the output fused in.
//
// The reference has no kernel for this layer: its Qwen3.5-like config is a description
// (configs/qwen35_35b_a3b.yaml:1-22) and a byte model (harness/synth.py:114-138). The algorithm is the published
// gated delta rule (Yang, Kautz, Hatamizadeh 2024): per value head, with a d_v x d_k state S,
//   S_t = a_t S_{t-1} (I - b_t k_t k_t^T) + b_t v_t k_t^T,    o_t = S_t q_t,
// k_t, q_t L2-normalised (q also scaled by d_k^-1/2), a_t = exp(g_t), g_t = -exp(A_log) softplus(a_raw + dt_bias),
// b_t = sigmoid(b_raw). Output: rmsnorm(o_t) * w * silu(z_t) over each head's d_v values (or o_t itself).
//
// Decode (HBM-bound: the fp32 state is read and written once): one CTA per (sequence, value head); every state
// row is independent, o_i = a (S_i . q) + u_i (k . q) with u_i = b (v_i - a S_i . k), S_i' = a S_i + u_i k.
// A row of 128 fp32 is 8 lanes x four 16-byte vectors, so one pass of a warp covers 4 rows, both dot products
// reduce over 8 lanes, and each lane keeps 8 vectors in flight.
//
// Prefill: one CTA per (sequence, value head) walks 64-token chunks. Within a chunk starting from S,
//   N_ij = b_i exp(cum_i - cum_j) k_i.k_j (j < i),  T = (I + N)^-1,  Qm_ij = exp(cum_i - cum_j) q_i.k_j (j <= i)
//   U^T = [b_i (v_i - exp(cum_i) S k_i)]^T T^T,      O^T = exp(cum_i) S Q^T + U^T Qm^T,
//   S'  = exp(cum_C) S + (U^T diag(exp(cum_C - cum_i))) K
// (the recurrence unrolled over the chunk; cum = running sum of g inside the chunk). Every contraction has the
// state's d_v rows as its M dimension, so each of the 8 warps owns 16 rows of S as mma accumulators for the whole
// walk and computes the matching 16 rows of P = S K^T, U^T, O^T and the update without exchanging anything;
// K K^T and Q K^T are split over the warps, and T is inverted in fp32 on the CUDA cores (16x16 diagonal blocks
// by forward substitution, then the blocks below by distance from the diagonal). Contractions are bf16
// mma.m16n8k16 with fp32 accumulation from ldmatrix'd, 128-byte-swizzled shared memory; the next chunk's
// q/k/v/z are loaded with cp.async under the current chunk's math.
#include "mmp_common.cuh"

namespace mmp {
namespace {

constexpr int GDK = 128;  // key head dim
constexpr int GDV = 128;  // value head dim

__device__ __forceinline__ float gdn_decay_log(float a_raw, float dt_bias, float A_log, bool has_A) {
  const float sp = softplus(a_raw + dt_bias);
  return -(has_A ? __expf(A_log) : 1.f) * sp;
}
__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// ============================================================================================ decode
struct GdnDecodeParams {
  float* state; int64_t s_line, s_head, s_row;  // [lines, nv, dv, dk] fp32
  const bf16* q; int64_t q_b, q_h;              // [B, nk, dk]
  const bf16* k; int64_t k_b, k_h;
  const bf16* v; int64_t v_b, v_h;              // [B, nv, dv]
  const bf16* a; int64_t a_b;                   // [B, nv] raw decay projection
  const bf16* b; int64_t b_b;                   // [B, nv] raw write-strength projection
  const float* A_log; const float* dt_bias;     // [nv] or null
  const bf16* z; int64_t z_b, z_h;              // [B, nv, dv] or null (no gate)
  const bf16* norm_w;                           // [dv] or null (output o itself)
  float eps;
  const int32_t* idx; int pad_slot;             // [B] state lines (null: line = row)
  bf16* out; int64_t o_b, o_h;                  // [B, nv, dv]
  int batch, nk, nv, lines;
  int* err;
};

constexpr int DEC_WARPS = 4;
constexpr int DEC_ROWS_WARP = GDV / DEC_WARPS;  // 32
constexpr int DEC_PASSES = DEC_ROWS_WARP / 4;   // 8 passes of 4 rows
constexpr int DEC_R = 2;                        // passes in flight

__device__ __forceinline__ void load_bf16x4(const bf16* p, float* f) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 x = unpack_bf16x2(u.x), y = unpack_bf16x2(u.y);
  f[0] = x.x; f[1] = x.y; f[2] = y.x; f[3] = y.y;
}

__global__ void __launch_bounds__(DEC_WARPS * 32) gdn_decode_kernel(const GdnDecodeParams P) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[DEC_WARPS];
  const int j = blockIdx.x, bq = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int li = lane & 7, sub = lane >> 3;  // lane in its row group, row group in the warp
  const int line = P.idx ? P.idx[bq] : bq;
  bf16* outp = P.out + bq * P.o_b + j * P.o_h;
  if (line == P.pad_slot) {
    if (tid < GDV) outp[tid] = f2bf(0.f);
    return;
  }
  if (line < 0 || line >= P.lines) {
    if (tid == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  float* st = P.state + line * P.s_line + j * P.s_head;
  const int row0 = warp * DEC_ROWS_WARP + sub;  // rows row0 + 4 p for passes p

  // two sets of DEC_R passes: the next set's loads are in flight while the current set is computed
  uint4 raw[2][DEC_R][4];
  auto load_rows = [&](uint4 (&dst)[DEC_R][4], int it) {
#pragma unroll
    for (int r = 0; r < DEC_R; ++r) {
      const int row = row0 + (it * DEC_R + r) * 4;
#pragma unroll
      for (int vv = 0; vv < 4; ++vv) dst[r][vv] = ld_stream16(st + row * P.s_row + (vv * 8 + li) * 4);
    }
  };
  load_rows(raw[0], 0);

  // q, k of the head's key head, this lane's 16 columns (vv * 8 + li) * 4 .. + 4, L2-normalised
  const int kh = j / (P.nv / P.nk);
  float qf[4][4], kf[4][4];
  float sq = 0.f, sk = 0.f;
#pragma unroll
  for (int vv = 0; vv < 4; ++vv) {
    const int c = (vv * 8 + li) * 4;
    load_bf16x4(P.q + bq * P.q_b + kh * P.q_h + c, qf[vv]);
    load_bf16x4(P.k + bq * P.k_b + kh * P.k_h + c, kf[vv]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sq = fmaf(qf[vv][e], qf[vv][e], sq);
      sk = fmaf(kf[vv][e], kf[vv][e], sk);
    }
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
    sk += __shfl_xor_sync(0xffffffffu, sk, o);
  }
  const float rq = rsqrtf(sq + 1e-6f) * rsqrtf(static_cast<float>(GDK)), rk = rsqrtf(sk + 1e-6f);
  float kq = 0.f;
#pragma unroll
  for (int vv = 0; vv < 4; ++vv)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      qf[vv][e] *= rq;
      kf[vv][e] *= rk;
      kq = fmaf(qf[vv][e], kf[vv][e], kq);
    }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) kq += __shfl_xor_sync(0xffffffffu, kq, o);

  const float g = gdn_decay_log(bf2f(P.a[bq * P.a_b + j]), P.dt_bias ? P.dt_bias[j] : 0.f,
                                P.A_log ? P.A_log[j] : 0.f, P.A_log != nullptr);
  const float dec = __expf(g);
  const float beta = sigmoidf_(bf2f(P.b[bq * P.b_b + j]));
  const bf16* vp = P.v + bq * P.v_b + j * P.v_h;

  float orow[DEC_PASSES];
#pragma unroll
  for (int it = 0; it < DEC_PASSES / DEC_R; ++it) {
    if (it + 1 < DEC_PASSES / DEC_R) load_rows(raw[(it + 1) & 1], it + 1);
#pragma unroll
    for (int r = 0; r < DEC_R; ++r) {
      const int row = row0 + (it * DEC_R + r) * 4;
      const uint4* cur = raw[it & 1][r];
      float s[4][4];
      float dk_ = 0.f, dq_ = 0.f;
#pragma unroll
      for (int vv = 0; vv < 4; ++vv) {
        s[vv][0] = __uint_as_float(cur[vv].x);
        s[vv][1] = __uint_as_float(cur[vv].y);
        s[vv][2] = __uint_as_float(cur[vv].z);
        s[vv][3] = __uint_as_float(cur[vv].w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          dk_ = fmaf(s[vv][e], kf[vv][e], dk_);
          dq_ = fmaf(s[vv][e], qf[vv][e], dq_);
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        dk_ += __shfl_xor_sync(0xffffffffu, dk_, o);
        dq_ += __shfl_xor_sync(0xffffffffu, dq_, o);
      }
      const float u = beta * (bf2f(vp[row]) - dec * dk_);
      orow[it * DEC_R + r] = fmaf(dec, dq_, u * kq);
#pragma unroll
      for (int vv = 0; vv < 4; ++vv) {
        float n[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) n[e] = fmaf(dec, s[vv][e], u * kf[vv][e]);
        st_stream16(st + row * P.s_row + (vv * 8 + li) * 4,
                    make_uint4(__float_as_uint(n[0]), __float_as_uint(n[1]), __float_as_uint(n[2]), __float_as_uint(n[3])));
      }
    }
  }

  float scale = 1.f;
  if (P.norm_w) {
    float ss = 0.f;
    if (li == 0) {
#pragma unroll
      for (int p = 0; p < DEC_PASSES; ++p) ss = fmaf(orow[p], orow[p], ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < DEC_WARPS; ++w) tot += red[w];
    scale = rsqrtf(tot / static_cast<float>(GDV) + P.eps);
  }
  if (li == 0) {
    const bf16* zp = P.z ? P.z + bq * P.z_b + j * P.z_h : nullptr;
#pragma unroll
    for (int p = 0; p < DEC_PASSES; ++p) {
      const int row = row0 + p * 4;
      float y = orow[p];
      if (P.norm_w) y = y * scale * bf2f(P.norm_w[row]);
      if (zp) y *= silu(bf2f(zp[row]));
      outp[row] = f2bf(y);
    }
  }
}

// ============================================================================================ prefill
constexpr int QC = 64;     // tokens per chunk
constexpr int THR = 256;   // 8 warps; warp w owns state rows 16 w .. 16 w + 15
constexpr int NLD = 68;    // fp32 row stride of the N / T scratch matrices
constexpr int XLD = 17;    // fp32 row stride of a 16 x 16 block product

struct GdnPrefillParams {
  const bf16* q; int64_t q_t, q_h;   // [T, nk, dk] (post-conv, not normalised)
  const bf16* k; int64_t k_t, k_h;
  const bf16* v; int64_t v_t, v_h;   // [T, nv, dv]
  const bf16* a; int64_t a_t;        // [T, nv] raw
  const bf16* b; int64_t b_t;        // [T, nv] raw
  const float* A_log; const float* dt_bias;
  const bf16* z; int64_t z_t, z_h;   // [T, nv, dv] or null
  const bf16* norm_w; float eps;     // [dv] or null
  float* state; int64_t s_line, s_head, s_row;
  const int32_t* cu_seqlens; const int32_t* state_idx; const int32_t* has_init;
  bf16* out; int64_t o_t, o_h;
  int nk, nv, lines;
  int* err;
};

struct GdnSmem {
  static constexpr int RB = 256;                   // bf16 row bytes of a [QC][128] tile
  static constexpr int TILE = QC * RB;             // 16 KB
  static constexpr int STAGE = 4 * TILE;           // q | k | v | z of one chunk
  static constexpr int N_OFF = 2 * STAGE;          // [QC][NLD] fp32: N
  static constexpr int TF_OFF = N_OFF + QC * NLD * 4;   // [QC][NLD] fp32: T while it is inverted
  static constexpr int X_OFF = TF_OFF + QC * NLD * 4;   // [3][16][XLD] fp32 block products
  static constexpr int T_OFF = X_OFF + 3 * 16 * XLD * 4 + 64;  // [QC][QC] bf16 T (row 128 bytes, swizzled)
  static constexpr int QM_OFF = T_OFF + QC * QC * 2;    // [QC][QC] bf16 Qm
  static constexpr int CUM_OFF = QM_OFF + QC * QC * 2;  // [QC] fp32 running log-decay
  static constexpr int GAM_OFF = CUM_OFF + QC * 4;      // [QC] exp(cum)
  static constexpr int BETA_OFF = GAM_OFF + QC * 4;     // [QC] beta
  static constexpr int W_OFF = BETA_OFF + QC * 4;       // [QC] exp(cum_C - cum)
  static constexpr int SQ_OFF = W_OFF + QC * 4;         // [8][QC] fp32 per-warp sums of squares of O
  static constexpr int BYTES = SQ_OFF + 8 * QC * 4;
  static_assert(X_OFF % 16 == 0 && T_OFF % 128 == 0 && QM_OFF % 128 == 0, "alignment");
};

__device__ __forceinline__ uint32_t sa(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
// 16-byte chunk c of row r in rows of `row_bytes` (a multiple of 128), XOR-swizzled inside each 128-byte group
__device__ __forceinline__ uint32_t swz(int r, int c, int row_bytes) { return r * row_bytes + ((c ^ (r & 7)) << 4); }

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

// A fragment (16 rows x k16) from two accumulator n8-tiles c0 (k 0..7) and c1 (k 8..15), each scaled per column
__device__ __forceinline__ void acc_to_a(const float* c0, const float* c1, uint32_t* a) {
  a[0] = pack_bf16x2(c0[0], c0[1]);
  a[1] = pack_bf16x2(c0[2], c0[3]);
  a[2] = pack_bf16x2(c1[0], c1[1]);
  a[3] = pack_bf16x2(c1[2], c1[3]);
}

// acc[8][4] (this warp's 16 rows x 64 tokens) += A (16 rows x 128, from the state accumulators) . X^T for a
// [QC][128] bf16 tile X (rows = tokens)
__device__ __forceinline__ void state_times_tileT(const float (*S)[4], uint32_t tile, int mat, int r8, float (*acc)[4]) {
#pragma unroll
  for (int kk = 0; kk < GDK / 16; ++kk) {
    uint32_t a[4];
    acc_to_a(S[2 * kk], S[2 * kk + 1], a);
#pragma unroll
    for (int np = 0; np < QC / 16; ++np) {
      uint32_t b[4];
      ldsm_x4(tile + swz(np * 16 + (mat >> 1) * 8 + r8, kk * 2 + (mat & 1), GdnSmem::RB), b);
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
}

// acc[8][4] += A (16 rows x 64 tokens, from accumulator tiles X[8][4]) . M^T for a [QC][QC] bf16 matrix M
__device__ __forceinline__ void tokens_times_matT(const float (*X)[4], uint32_t m, int mat, int r8, float (*acc)[4]) {
#pragma unroll
  for (int kk = 0; kk < QC / 16; ++kk) {
    uint32_t a[4];
    acc_to_a(X[2 * kk], X[2 * kk + 1], a);
#pragma unroll
    for (int np = 0; np < QC / 16; ++np) {
      uint32_t b[4];
      ldsm_x4(m + swz(np * 16 + (mat >> 1) * 8 + r8, kk * 2 + (mat & 1), QC * 2), b);
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
}

__global__ void __launch_bounds__(THR, 1) gdn_prefill_kernel(const GdnPrefillParams P) {
  using L = GdnSmem;
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_trigger();
  pdl_wait();
  const int j = blockIdx.x, seq = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3, mat = lane >> 3, r8 = lane & 7;
  const int t_begin = P.cu_seqlens[seq], t_end = P.cu_seqlens[seq + 1];
  const int line = P.state_idx[seq];
  if (line < 0 || line >= P.lines) {
    if (tid == 0) flag_error(P.err, DEVERR_INDEX);
    return;
  }
  const int kh = j / (P.nv / P.nk);
  const bool has_A = P.A_log != nullptr;
  const float A_log = has_A ? P.A_log[j] : 0.f, dtb = P.dt_bias ? P.dt_bias[j] : 0.f;
  float* sN = reinterpret_cast<float*>(smem + L::N_OFF);
  float* sTf = reinterpret_cast<float*>(smem + L::TF_OFF);
  float* sX = reinterpret_cast<float*>(smem + L::X_OFF);
  float* sCum = reinterpret_cast<float*>(smem + L::CUM_OFF);
  float* sGam = reinterpret_cast<float*>(smem + L::GAM_OFF);
  float* sBeta = reinterpret_cast<float*>(smem + L::BETA_OFF);
  float* sW = reinterpret_cast<float*>(smem + L::W_OFF);
  float* sSq = reinterpret_cast<float*>(smem + L::SQ_OFF);
  const uint32_t base = sa(smem);
  const uint32_t sT = base + L::T_OFF, sQm = base + L::QM_OFF;
  float* gstate = P.state + line * P.s_line + j * P.s_head;
  const int vr0 = warp * 16;  // this warp's state rows

  // ---- initial state: accumulator (row vr0 + g + 8 (e >> 1), column nt * 8 + 2 tq + (e & 1))
  float S[GDK / 8][4];
  {
    const bool init = P.has_init && P.has_init[seq];
#pragma unroll
    for (int nt = 0; nt < GDK / 8; ++nt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = vr0 + g + h * 8, c = nt * 8 + 2 * tq;
        float2 v = make_float2(0.f, 0.f);
        if (init) v = *reinterpret_cast<const float2*>(gstate + r * P.s_row + c);
        S[nt][2 * h] = v.x;
        S[nt][2 * h + 1] = v.y;
      }
    }
  }

  auto issue = [&](int c0, int stage) {
    const int qn = min(QC, t_end - c0);
    const uint32_t sQ = base + stage * L::STAGE, sK = sQ + L::TILE, sV = sK + L::TILE, sZ = sV + L::TILE;
    for (int i = tid; i < QC * 16; i += THR) {
      const int r = i >> 4, c = i & 15;
      const bool ok = r < qn;
      const int64_t t = c0 + (ok ? r : 0);
      cp16(sQ + swz(r, c, L::RB), P.q + t * P.q_t + kh * P.q_h + c * 8, ok);
      cp16(sK + swz(r, c, L::RB), P.k + t * P.k_t + kh * P.k_h + c * 8, ok);
      cp16(sV + swz(r, c, L::RB), P.v + t * P.v_t + j * P.v_h + c * 8, ok);
      if (P.z) cp16(sZ + swz(r, c, L::RB), P.z + t * P.z_t + j * P.z_h + c * 8, ok);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };
  float anext[2] = {0.f, 0.f}, bnext[2] = {0.f, 0.f};  // warp 0: raw gates of tokens 2 lane, 2 lane + 1
  auto load_gates = [&](int c0) {
    if (warp == 0) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = lane * 2 + e;
        const bool ok = c0 + r < t_end;
        anext[e] = ok ? bf2f(P.a[static_cast<int64_t>(c0 + r) * P.a_t + j]) : 0.f;
        bnext[e] = ok ? bf2f(P.b[static_cast<int64_t>(c0 + r) * P.b_t + j]) : 0.f;
      }
    }
  };
  if (t_begin < t_end) {
    issue(t_begin, 0);
    load_gates(t_begin);
  }

  int stage = 0;
  for (int c0 = t_begin; c0 < t_end; c0 += QC, stage ^= 1) {
    const int qn = min(QC, t_end - c0);
    if (warp == 0) {
      // g, beta of tokens 2 lane, 2 lane + 1 (zero past the sequence end) and the inclusive running sum of g
      float gg[2], bb[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = lane * 2 + e < qn;
        gg[e] = ok ? gdn_decay_log(anext[e], dtb, A_log, has_A) : 0.f;
        bb[e] = ok ? sigmoidf_(bnext[e]) : 0.f;
      }
      const float c1 = gg[0] + gg[1];
      float run = c1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, run, o);
        if (lane >= o) run += v;
      }
      const float total = __shfl_sync(0xffffffffu, run, 31);
      const float cs[2] = {run - c1 + gg[0], run};
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = lane * 2 + e;
        sCum[r] = cs[e];
        sGam[r] = __expf(cs[e]);
        sBeta[r] = bb[e];
        sW[r] = __expf(total - cs[e]);
      }
    }
    if (c0 + QC < t_end) {
      issue(c0 + QC, stage ^ 1);
      load_gates(c0 + QC);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();
    const uint32_t sQ = base + stage * L::STAGE, sK = sQ + L::TILE;
    uint8_t* pQ = smem + stage * L::STAGE;

    // ---- L2-normalise the q and k rows in place (q also times d_k^-1/2): 16 lanes per row
    {
      const int hl = lane >> 4, c = lane & 15;
#pragma unroll
      for (int p = 0; p < 2 * QC / 16; ++p) {
        const int job = p * 16 + warp * 2 + hl;  // 0..127: q rows then k rows
        const int m = job >> 6, r = job & (QC - 1);
        uint4* ptr = reinterpret_cast<uint4*>(pQ + m * L::TILE + swz(r, c, L::RB));
        const uint4 u = *ptr;
        float f[8];
        const float2 x0 = unpack_bf16x2(u.x), x1 = unpack_bf16x2(u.y), x2 = unpack_bf16x2(u.z), x3 = unpack_bf16x2(u.w);
        f[0] = x0.x; f[1] = x0.y; f[2] = x1.x; f[3] = x1.y; f[4] = x2.x; f[5] = x2.y; f[6] = x3.x; f[7] = x3.y;
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float sc = rsqrtf(ss + 1e-6f) * (m == 0 ? rsqrtf(static_cast<float>(GDK)) : 1.f);
        *ptr = make_uint4(pack_bf16x2(f[0] * sc, f[1] * sc), pack_bf16x2(f[2] * sc, f[3] * sc),
                          pack_bf16x2(f[4] * sc, f[5] * sc), pack_bf16x2(f[6] * sc, f[7] * sc));
      }
    }
    __syncthreads();

    // ---- K K^T and Q K^T: warp owns rows i = r0 .. r0 + 15, columns j = s0 .. s0 + 31
    {
      const int r0 = (warp >> 1) * 16, s0 = (warp & 1) * 32;
      float kk_[4][4] = {}, qk_[4][4] = {};
#pragma unroll 2
      for (int kc = 0; kc < GDK / 16; ++kc) {
        uint32_t ak[4], aq[4], b[2][4];
        ldsm_x4(sK + swz(r0 + (mat & 1) * 8 + r8, kc * 2 + (mat >> 1), L::RB), ak);
        ldsm_x4(sQ + swz(r0 + (mat & 1) * 8 + r8, kc * 2 + (mat >> 1), L::RB), aq);
#pragma unroll
        for (int np = 0; np < 2; ++np)
          ldsm_x4(sK + swz(s0 + np * 16 + (mat >> 1) * 8 + r8, kc * 2 + (mat & 1), L::RB), b[np]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          mma16816(kk_[nt], ak, b[nt >> 1][(nt & 1) * 2], b[nt >> 1][(nt & 1) * 2 + 1]);
          mma16816(qk_[nt], aq, b[nt >> 1][(nt & 1) * 2], b[nt >> 1][(nt & 1) * 2 + 1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = r0 + g + h * 8, c = s0 + nt * 8 + 2 * tq;
          const float ci = sCum[i], bi = sBeta[i];
          float n[2], m[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int jj = c + e;
            const float ratio = jj <= i ? __expf(ci - sCum[jj]) : 0.f;
            n[e] = jj < i ? bi * ratio * kk_[nt][2 * h + e] : 0.f;
            m[e] = ratio * qk_[nt][2 * h + e];
          }
          *reinterpret_cast<float2*>(sN + i * NLD + c) = make_float2(n[0], n[1]);
          *reinterpret_cast<uint32_t*>(smem + L::QM_OFF + swz(i, c >> 3, QC * 2) + (c & 7) * 2) = pack_bf16x2(m[0], m[1]);
        }
      }
    }
    __syncthreads();

    // ---- T = (I + N)^-1 in fp32: diagonal 16x16 blocks, one column per thread (threads 0..63)
    if (tid < 64) {
      const int d = tid >> 4, e = tid & 15, o = d * 16;
      float t[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) t[i] = i == e ? 1.f : 0.f;
#pragma unroll
      for (int i = 1; i < 16; ++i) {
        if (i > e) {
          float s = 0.f;
#pragma unroll
          for (int jj = 0; jj < i; ++jj)
            if (jj >= e) s = fmaf(sN[(o + i) * NLD + o + jj], t[jj], s);
          t[i] = -s;
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) sTf[(o + i) * NLD + o + e] = t[i];
    }
    __syncthreads();
    // blocks below the diagonal, by distance: X = sum_{bj <= kb < bi} N_{bi,kb} T_{kb,bj}; T_{bi,bj} = -T_{bi,bi} X
#pragma unroll 1
    for (int dist = 1; dist < 4; ++dist) {
      const int nblk = 4 - dist;
      for (int idx = tid; idx < nblk * 256; idx += THR) {
        const int bj = idx >> 8, r = (idx >> 4) & 15, c = idx & 15, bi = bj + dist;
        float x = 0.f;
        for (int kb = bj; kb < bi; ++kb) {
#pragma unroll
          for (int m = 0; m < 16; ++m) x = fmaf(sN[(bi * 16 + r) * NLD + kb * 16 + m], sTf[(kb * 16 + m) * NLD + bj * 16 + c], x);
        }
        sX[(bj * 16 + r) * XLD + c] = x;
      }
      __syncthreads();
      for (int idx = tid; idx < nblk * 256; idx += THR) {
        const int bj = idx >> 8, r = (idx >> 4) & 15, c = idx & 15, bi = bj + dist;
        float x = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (m <= r) x = fmaf(sTf[(bi * 16 + r) * NLD + bi * 16 + m], sX[(bj * 16 + m) * XLD + c], x);
        sTf[(bi * 16 + r) * NLD + bj * 16 + c] = -x;
      }
      __syncthreads();
    }
    // bf16 copy of T (zero above the block diagonal)
    for (int idx = tid; idx < QC * QC / 2; idx += THR) {
      const int i = idx >> 5, c = (idx & 31) * 2;
      float2 v = make_float2(0.f, 0.f);
      if ((c >> 4) <= (i >> 4)) v = *reinterpret_cast<const float2*>(sTf + i * NLD + c);
      *reinterpret_cast<uint32_t*>(smem + L::T_OFF + swz(i, c >> 3, QC * 2) + (c & 7) * 2) = pack_bf16x2(v.x, v.y);
    }
    __syncthreads();

    // ---- this warp's 16 state rows: P = S K^T, R^T, U^T = R^T T^T, O^T, S update
    float U[QC / 8][4];
    {
      float Pm[QC / 8][4] = {};
      state_times_tileT(S, sK, mat, r8, Pm);
      // R^T[v][i] = beta_i (V[i][v] - exp(cum_i) P[v][i])
#pragma unroll
      for (int nt = 0; nt < QC / 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = nt * 8 + 2 * tq + (e & 1), v = vr0 + g + (e >> 1) * 8;
          const float vv = bf2f(*reinterpret_cast<const bf16*>(smem + stage * L::STAGE + 2 * L::TILE + swz(i, v >> 3, L::RB) +
                                                               (v & 7) * 2));
          Pm[nt][e] = sBeta[i] * (vv - sGam[i] * Pm[nt][e]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < QC / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) U[nt][e] = 0.f;
      tokens_times_matT(Pm, sT, mat, r8, U);
    }
    float O[QC / 8][4] = {};
    state_times_tileT(S, sQ, mat, r8, O);
#pragma unroll
    for (int nt = 0; nt < QC / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) O[nt][e] *= sGam[nt * 8 + 2 * tq + (e & 1)];
    }
    tokens_times_matT(U, sQm, mat, r8, O);
    {
      const float decC = sGam[QC - 1];
#pragma unroll
      for (int nt = 0; nt < GDK / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[nt][e] *= decC;
#pragma unroll
      for (int kc = 0; kc < QC / 16; ++kc) {
        const int i0 = kc * 16 + 2 * tq;
        const float w0 = sW[i0], w1 = sW[i0 + 1], w8 = sW[i0 + 8], w9 = sW[i0 + 9];
        uint32_t a[4];
        a[0] = pack_bf16x2(U[2 * kc][0] * w0, U[2 * kc][1] * w1);
        a[1] = pack_bf16x2(U[2 * kc][2] * w0, U[2 * kc][3] * w1);
        a[2] = pack_bf16x2(U[2 * kc + 1][0] * w8, U[2 * kc + 1][1] * w9);
        a[3] = pack_bf16x2(U[2 * kc + 1][2] * w8, U[2 * kc + 1][3] * w9);
#pragma unroll
        for (int np = 0; np < GDK / 16; ++np) {
          uint32_t b[4];  // K[i][c]: transposed load gives (k = i, n = c) fragments for n-tiles 2 np, 2 np + 1
          ldsm_x4_t(sK + swz(kc * 16 + (mat & 1) * 8 + r8, np * 2 + (mat >> 1), L::RB), b);
          mma16816(S[2 * np], a, b[0], b[1]);
          mma16816(S[2 * np + 1], a, b[2], b[3]);
        }
      }
    }

    // ---- output: per-token RMS over the head's d_v values (partials per warp), gate, stage into the z tile
    if (P.norm_w) {
#pragma unroll
      for (int nt = 0; nt < QC / 8; ++nt) {
        float c0s = O[nt][0] * O[nt][0] + O[nt][2] * O[nt][2];
        float c1s = O[nt][1] * O[nt][1] + O[nt][3] * O[nt][3];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          c0s += __shfl_xor_sync(0xffffffffu, c0s, o);
          c1s += __shfl_xor_sync(0xffffffffu, c1s, o);
        }
        if (g == 0) *reinterpret_cast<float2*>(sSq + warp * QC + nt * 8 + 2 * tq) = make_float2(c0s, c1s);
      }
    }
    __syncthreads();
    const float w_lo = P.norm_w ? bf2f(P.norm_w[vr0 + g]) : 1.f, w_hi = P.norm_w ? bf2f(P.norm_w[vr0 + g + 8]) : 1.f;
#pragma unroll
    for (int nt = 0; nt < QC / 8; ++nt) {
      float rs[2] = {1.f, 1.f};
      if (P.norm_w) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float tot = 0.f;
#pragma unroll
          for (int w = 0; w < 8; ++w) tot += sSq[w * QC + nt * 8 + 2 * tq + e];
          rs[e] = rsqrtf(tot / static_cast<float>(GDV) + P.eps);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = nt * 8 + 2 * tq + (e & 1), v = vr0 + g + (e >> 1) * 8;
        bf16* zo = reinterpret_cast<bf16*>(smem + stage * L::STAGE + 3 * L::TILE + swz(i, v >> 3, L::RB) + (v & 7) * 2);
        float y = O[nt][e] * rs[e & 1] * ((e >> 1) ? w_hi : w_lo);
        if (P.z) y *= silu(bf2f(*zo));
        *zo = f2bf(y);
      }
    }
    __syncthreads();
    for (int idx = tid; idx < QC * 16; idx += THR) {
      const int i = idx >> 4, c = idx & 15;
      if (i < qn)
        st16(P.out + static_cast<int64_t>(c0 + i) * P.o_t + j * P.o_h + c * 8,
             *reinterpret_cast<const uint4*>(smem + stage * L::STAGE + 3 * L::TILE + swz(i, c, L::RB)));
    }
    __syncthreads();  // the stage and the per-chunk scalars are rewritten by the next chunk
  }

  // ---- final state -> the sequence's line
#pragma unroll
  for (int nt = 0; nt < GDK / 8; ++nt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = vr0 + g + h * 8, c = nt * 8 + 2 * tq;
      *reinterpret_cast<float2*>(gstate + r * P.s_row + c) = make_float2(S[nt][2 * h], S[nt][2 * h + 1]);
    }
  }
}

}  // namespace
}  // namespace mmp

using namespace mmp;

extern "C" int mmp_gdn_decode(float* state, int64_t s_line, int64_t s_head, int64_t s_row,
                              const void* q, int64_t q_b, int64_t q_h, const void* k, int64_t k_b, int64_t k_h,
                              const void* v, int64_t v_b, int64_t v_h, const void* a, int64_t a_b,
                              const void* b, int64_t b_b, const float* A_log, const float* dt_bias,
                              const void* z, int64_t z_b, int64_t z_h, const void* norm_w, float eps,
                              const int32_t* idx, int pad_slot, void* out, int64_t o_b, int64_t o_h,
                              int batch, int nk, int nv, int dk, int dv, int lines, int* err, void* stream) {
  if (batch == 0) return MMP_OK;
  if (!state || !q || !k || !v || !a || !b || !out)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_decode: null pointer");
  if (batch < 0 || batch > 65535 || nk <= 0 || nv <= 0 || nv % nk || lines <= 0 || nv > 65535)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_decode: bad sizes batch=%d nk=%d nv=%d lines=%d", batch, nk, nv, lines);
  if (dk != GDK || dv != GDV)
    return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_gdn_decode: head dims %d x %d (only 128 x 128)", dk, dv);
  if (!aligned16(state) || s_line % 4 || s_head % 4 || s_row % 4)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_decode: state rows must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k)) % 8 || q_b % 4 || q_h % 4 || k_b % 4 || k_h % 4)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_decode: q/k rows must be 8-byte aligned");
  GdnDecodeParams P{state, s_line, s_head, s_row,
                    static_cast<const bf16*>(q), q_b, q_h, static_cast<const bf16*>(k), k_b, k_h,
                    static_cast<const bf16*>(v), v_b, v_h, static_cast<const bf16*>(a), a_b,
                    static_cast<const bf16*>(b), b_b, A_log, dt_bias,
                    static_cast<const bf16*>(z), z_b, z_h, static_cast<const bf16*>(norm_w), eps,
                    idx, pad_slot, static_cast<bf16*>(out), o_b, o_h, batch, nk, nv, lines, err};
  cudaError_t e = mmp::launch(gdn_decode_kernel, dim3(nv, batch), dim3(DEC_WARPS * 32), 0,
                              static_cast<cudaStream_t>(stream), nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gdn_decode: launch failed: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_gdn_decode");
}

extern "C" int mmp_gdn_prefill(const void* q, int64_t q_t, int64_t q_h, const void* k, int64_t k_t, int64_t k_h,
                               const void* v, int64_t v_t, int64_t v_h, const void* a, int64_t a_t,
                               const void* b, int64_t b_t, const float* A_log, const float* dt_bias,
                               const void* z, int64_t z_t, int64_t z_h, const void* norm_w, float eps,
                               float* state, int64_t s_line, int64_t s_head, int64_t s_row,
                               const int32_t* cu_seqlens, const int32_t* state_idx, const int32_t* has_init,
                               void* out, int64_t o_t, int64_t o_h,
                               int nseq, int ntok, int nk, int nv, int dk, int dv, int lines, int* err, void* stream) {
  if (nseq == 0) return MMP_OK;
  if (!q || !k || !v || !a || !b || !state || !cu_seqlens || !state_idx || !out)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill: null pointer");
  if (nseq < 0 || nseq > 65535 || ntok < 0 || nk <= 0 || nv <= 0 || nv % nk || nv > 65535 || lines <= 0)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill: bad sizes nseq=%d nk=%d nv=%d lines=%d", nseq, nk, nv, lines);
  if (dk != GDK || dv != GDV)
    return mmp_set_error(MMP_ERR_UNSUPPORTED, "mmp_gdn_prefill: head dims %d x %d (only 128 x 128)", dk, dv);
  const bool zal = !z || (aligned16(z) && z_t % 8 == 0 && z_h % 8 == 0);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !zal || q_t % 8 || q_h % 8 || k_t % 8 ||
      k_h % 8 || v_t % 8 || v_h % 8 || o_t % 8 || o_h % 8)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill: q, k, v, z and out rows must be 16-byte aligned");
  if (!aligned16(state) || s_line % 4 || s_head % 4 || s_row % 4)
    return mmp_set_error(MMP_ERR_INVALID, "mmp_gdn_prefill: state rows must be 16-byte aligned");
  GdnPrefillParams P{static_cast<const bf16*>(q), q_t, q_h, static_cast<const bf16*>(k), k_t, k_h,
                     static_cast<const bf16*>(v), v_t, v_h, static_cast<const bf16*>(a), a_t,
                     static_cast<const bf16*>(b), b_t, A_log, dt_bias,
                     static_cast<const bf16*>(z), z_t, z_h, static_cast<const bf16*>(norm_w), eps,
                     state, s_line, s_head, s_row, cu_seqlens, state_idx, has_init,
                     static_cast<bf16*>(out), o_t, o_h, nk, nv, lines, err};
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gdn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GdnSmem::BYTES);
    if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gdn_prefill: smem attribute: %s", cudaGetErrorString(e));
    attr[dev] = true;
  }
  cudaError_t e = mmp::launch(gdn_prefill_kernel, dim3(nv, nseq), dim3(THR), GdnSmem::BYTES,
                              static_cast<cudaStream_t>(stream), nullptr, 0, P);
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "mmp_gdn_prefill: launch failed: %s", cudaGetErrorString(e));
  return mmp_check_launch("mmp_gdn_prefill");
}
