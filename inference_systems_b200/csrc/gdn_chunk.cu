// Chunked Gated DeltaNet prefill.
//
// The token-recurrent scan (gdn.cu) walks every prompt token in order inside
// one CTA per (head, sequence).  For long prompts that chain dominates the
// prefill, so prefill runs the chunk form of the gated delta rule instead
// (the WY/UT representation of Yang et al., "Parallelizing Linear Transformers
// with the Delta Rule over Sequence Length", NeurIPS 2024, and "Gated Delta
// Networks", ICLR 2025), derived here for this engine's state layout
// S[key][value]:
//
//   per token   S_t = e^{g_t} S_{t-1} + k_t d_t^T,  d_t = b_t (v_t - e^{g_t} S_{t-1}^T k_t),
//               o_t = S_t^T q_t
//   chunk of n tokens from state S0, G_t = g_1 + ... + g_t (within the chunk):
//               A_tj = b_t e^{G_t - G_j} (k_t . k_j)          (j < t)
//               T    = (I + A)^{-1}                            (forward substitution)
//               U = T (b * V),  W = T (b e^{G} * K),  D = U - W S0
//               O = (e^{G} * Q) S0 + P D,   P_tj = e^{G_t - G_j} (q_t . k_j)  (j <= t)
//               S_n = e^{G_n} S0 + (e^{G_n - G} * K)^T D
//
// gdn_chunk_prep_kernel: one CTA per (chunk, value head), all chunks in
//   parallel: causal conv + SiLU, L2 norms, beta/decay, and everything above
//   that does not depend on S0 (W, U, e^G Q, e^{G_n-G} K, P, e^{G_n}).
// gdn_chunk_state_kernel: one CTA per (32 value columns, value head, sequence)
//   carries its slice of S through the sequence's chunks in order (value
//   columns of the state evolve independently), writes the pre-norm output
//   and the final state, and commits the new conv window.
// gdn_chunk_norm_kernel: gated RMSNorm of each (token, head) row.
// All arithmetic is fp32; the projection input is bf16 as in the scan.

#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "launch.cuh"

namespace isb {
namespace {

constexpr int D = 128;        // key / value head dim
constexpr int KW = 4;         // causal conv width
constexpr int CL = 64;        // chunk length
constexpr int LDR = D + 4;    // padded row stride (floats) of [CL][D] tiles
constexpr int LDC = CL + 1;   // padded row stride of [CL][CL] tiles
constexpr int SLICE = 32;     // value columns per state CTA
constexpr int LDS = SLICE + 4;
// workspace floats per (chunk, value head): W, U, Qt, Kt [CL][D]; P [CL][CL]; gamma
constexpr int WS_W = 0, WS_U = CL * D, WS_Q = 2 * CL * D, WS_K = 3 * CL * D, WS_P = 4 * CL * D,
              WS_G = 4 * CL * D + CL * CL, WS_STRIDE = 4 * CL * D + CL * CL + 4;

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

struct ChunkArgs {
  const __nv_bfloat16* proj;
  int proj_stride;
  const int* chunk_seq;   // [nc]
  const int* chunk_t0;    // [nc] first row of the chunk
  const int* chunk_n;     // [nc] rows in the chunk (1..CL)
  const int* cu_chunks;   // [B+1]
  const int* cu_seqlens;  // [B+1]
  const int* slots;       // [B]
  const __nv_bfloat16* conv_w;  // [C, 4]
  const float* A_log;
  const float* dt_bias;
  const __nv_bfloat16* norm_w;
  float* rec;             // [S, Hv, D, D]
  __nv_bfloat16* conv;    // [S, C, 3]
  float* ws;              // [nc, Hv, WS_STRIDE]
  float* o32;             // [T, Hv, D] pre-norm output
  __nv_bfloat16* out;     // [T, Hv * D]
  int Hk, Hv, C, T;
  float eps;
};

constexpr int kPrepSmemFloats = 3 * CL * LDR + 2 * CL * LDC + 3 * CL;
constexpr int kStateSmemFloats = 3 * CL * LDR + CL * LDC + 2 * CL * LDS + D * LDS;

__global__ void __launch_bounds__(256) gdn_chunk_prep_kernel(ChunkArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm[];
  float* q_s = sm;                    // [CL][LDR]
  float* k_s = q_s + CL * LDR;        // [CL][LDR]
  float* v_s = k_s + CL * LDR;        // [CL][LDR]
  float* kk = v_s + CL * LDR;         // [CL][LDC]   k.k, then A
  float* qk = kk + CL * LDC;          // [CL][LDC]   q.k
  float* beta_s = qk + CL * LDC;      // [CL]
  float* g_s = beta_s + CL;           // [CL]
  float* G_s = g_s + CL;              // [CL]

  const int c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s = a.chunk_seq[c], t0 = a.chunk_t0[c], n = a.chunk_n[c];
  const int seq0 = a.cu_seqlens[s], slot = a.slots[s];
  const int r = a.Hv / a.Hk, hk = h / r;
  const int kd = a.Hk * D;
  // ---- causal conv + SiLU: thread -> q (tid < 128) or k channel, and a v channel (tid < 128)
  const int qk_ch = tid < 128 ? hk * D + tid : kd + hk * D + (tid - 128);
  const int v_ch = 2 * kd + h * D + (tid & 127);
  float wq[KW], wv[KW];
#pragma unroll
  for (int i = 0; i < KW; ++i) {
    wq[i] = bf(a.conv_w[qk_ch * KW + i]);
    wv[i] = tid < 128 ? bf(a.conv_w[v_ch * KW + i]) : 0.f;
  }
  auto X = [&](int ch, int row) -> float {  // raw input of channel ch at row (earlier rows: conv state)
    if (row >= seq0) return bf(a.proj[size_t(row) * a.proj_stride + ch]);
    return bf(a.conv[(size_t(slot) * a.C + ch) * (KW - 1) + (KW - 1) - (seq0 - row)]);
  };
  float* qk_dst = tid < 128 ? q_s + tid : k_s + (tid - 128);
  for (int i = 0; i < CL; ++i) {
    float yq = 0.f, yv = 0.f;
    if (i < n) {
      const int t = t0 + i;
#pragma unroll
      for (int w = 0; w < KW; ++w) yq += wq[w] * X(qk_ch, t - (KW - 1) + w);
      yq = silu_f(yq);
      if (tid < 128) {
#pragma unroll
        for (int w = 0; w < KW; ++w) yv += wv[w] * X(v_ch, t - (KW - 1) + w);
        yv = silu_f(yv);
      }
    }
    qk_dst[i * LDR] = yq;
    if (tid < 128) v_s[i * LDR + tid] = yv;
  }
  if (tid < CL) {
    float b = 0.f, g = 0.f;
    if (tid < n) {
      const __nv_bfloat16* row = a.proj + size_t(t0 + tid) * a.proj_stride + a.C + a.Hv * D;
      b = 1.f / (1.f + __expf(-bf(row[h])));
      g = -__expf(a.A_log[h]) * softplus_f(bf(row[a.Hv + h]) + a.dt_bias[h]);
    }
    beta_s[tid] = b;
    g_s[tid] = g;
  }
  __syncthreads();
  // ---- L2 norms per row (q also scaled by 1/sqrt(D)); cumulative log decay
  const float inv_sqrt_d = rsqrtf(float(D));
  for (int i = warp; i < n; i += 8) {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x = q_s[i * LDR + lane + 32 * e], y = k_s[i * LDR + lane + 32 * e];
      sq += x * x;
      sk += y * y;
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    const float iq = rsqrtf(sq + 1e-6f) * inv_sqrt_d, ik = rsqrtf(sk + 1e-6f);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      q_s[i * LDR + lane + 32 * e] *= iq;
      k_s[i * LDR + lane + 32 * e] *= ik;
    }
  }
  if (warp == 0) {  // inclusive prefix sum of g over the 64 rows (2 per lane)
    float x0 = g_s[2 * lane], x1 = g_s[2 * lane + 1];
    float v = x0 + x1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    const float before = v - (x0 + x1);
    G_s[2 * lane] = before + x0;
    G_s[2 * lane + 1] = v;
  }
  __syncthreads();
  // ---- k.k and q.k (64 x 64): each thread a 4 x 4 block
  {
    const int bi = (tid >> 4) * 4, bj = (tid & 15) * 4;
    float akk[4][4] = {}, aqk[4][4] = {};
    for (int d = 0; d < D; d += 4) {
      float4 kr[4], qr[4], kc[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        kr[x] = *reinterpret_cast<const float4*>(k_s + (bi + x) * LDR + d);
        qr[x] = *reinterpret_cast<const float4*>(q_s + (bi + x) * LDR + d);
        kc[x] = *reinterpret_cast<const float4*>(k_s + (bj + x) * LDR + d);
      }
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          akk[x][y] += kr[x].x * kc[y].x + kr[x].y * kc[y].y + kr[x].z * kc[y].z + kr[x].w * kc[y].w;
          aqk[x][y] += qr[x].x * kc[y].x + qr[x].y * kc[y].y + qr[x].z * kc[y].z + qr[x].w * kc[y].w;
        }
    }
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) {
        kk[(bi + x) * LDC + bj + y] = akk[x][y];
        qk[(bi + x) * LDC + bj + y] = aqk[x][y];
      }
  }
  __syncthreads();
  // ---- chunk-local outputs that need no forward substitution
  float* ws = a.ws + (size_t(c) * a.Hv + h) * WS_STRIDE;
  const float Gn = G_s[n - 1];
  for (int idx = tid; idx < CL * D; idx += 256) {
    const int i = idx / D, d = idx % D;
    const bool ok = i < n;
    ws[WS_Q + idx] = ok ? __expf(G_s[i]) * q_s[i * LDR + d] : 0.f;
    ws[WS_K + idx] = ok ? __expf(Gn - G_s[i]) * k_s[i * LDR + d] : 0.f;
  }
  for (int idx = tid; idx < CL * CL; idx += 256) {
    const int i = idx / CL, j = idx % CL;
    ws[WS_P + idx] = (i < n && j <= i) ? __expf(G_s[i] - G_s[j]) * qk[i * LDC + j] : 0.f;
  }
  if (tid == 0) ws[WS_G] = __expf(Gn);
  __syncthreads();
  // ---- A (strictly lower) in place of k.k; right-hand sides R = [b * V | b e^G * K]
  for (int idx = tid; idx < CL * CL; idx += 256) {
    const int i = idx / CL, j = idx % CL;
    kk[i * LDC + j] = (i < n && j < i) ? beta_s[i] * __expf(G_s[i] - G_s[j]) * kk[i * LDC + j] : 0.f;
  }
  for (int idx = tid; idx < CL * D; idx += 256) {
    const int i = idx / D, d = idx % D;
    v_s[i * LDR + d] *= beta_s[i];
    k_s[i * LDR + d] *= beta_s[i] * __expf(G_s[i]);
  }
  __syncthreads();
  // ---- forward substitution X_i = R_i - sum_{j<i} A_ij X_j: thread = one of the 256 columns
  {
    float* col = tid < 128 ? v_s + tid : k_s + (tid - 128);
    for (int i = 1; i < n; ++i) {
      float acc = col[i * LDR];
      const float* arow = kk + i * LDC;
      for (int j = 0; j < i; ++j) acc -= arow[j] * col[j * LDR];
      col[i * LDR] = acc;
    }
  }
  __syncthreads();
  for (int idx = tid; idx < CL * D; idx += 256) {
    const int i = idx / D, d = idx % D;
    ws[WS_U + idx] = v_s[i * LDR + d];
    ws[WS_W + idx] = k_s[i * LDR + d];
  }
}

__global__ void __launch_bounds__(256) gdn_chunk_state_kernel(ChunkArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float sm[];
  float* W_s = sm;                    // [CL][LDR]
  float* Q_s = W_s + CL * LDR;        // [CL][LDR]
  float* K_s = Q_s + CL * LDR;        // [CL][LDR]
  float* P_s = K_s + CL * LDR;        // [CL][LDC]
  float* U_s = P_s + CL * LDC;        // [CL][LDS]
  float* Dl_s = U_s + CL * LDS;       // [CL][LDS]
  float* S_s = Dl_s + CL * LDS;       // [D][LDS]

  const int sv = blockIdx.x, h = blockIdx.y, s = blockIdx.z, tid = threadIdx.x;
  const int c0 = a.cu_chunks[s], c1 = a.cu_chunks[s + 1];
  const int slot = a.slots[s];
  const int col0 = sv * SLICE;
  float* S = a.rec + ((size_t(slot) * a.Hv + h) * D) * D;
  for (int idx = tid; idx < D * SLICE; idx += 256) {
    const int d = idx / SLICE, cc = idx % SLICE;
    S_s[d * LDS + cc] = S[d * D + col0 + cc];
  }
  // thread layouts: (row i = tid / 4, 8 columns) for n x 32 outputs; (row d = tid / 2, 16 columns) for the state
  const int oi = tid >> 2, oc = (tid & 3) * 8;
  const int sd = tid >> 1, sc = (tid & 1) * 16;
  for (int c = c0; c < c1; ++c) {
    const int n = a.chunk_n[c], t0 = a.chunk_t0[c];
    const float* ws = a.ws + (size_t(c) * a.Hv + h) * WS_STRIDE;
    __syncthreads();  // previous chunk's readers are done with the tiles
    for (int idx = tid; idx < n * (D / 4); idx += 256) {
      const int i = idx / (D / 4), d4 = (idx % (D / 4)) * 4;
      *reinterpret_cast<float4*>(W_s + i * LDR + d4) = *reinterpret_cast<const float4*>(ws + WS_W + i * D + d4);
      *reinterpret_cast<float4*>(Q_s + i * LDR + d4) = *reinterpret_cast<const float4*>(ws + WS_Q + i * D + d4);
      *reinterpret_cast<float4*>(K_s + i * LDR + d4) = *reinterpret_cast<const float4*>(ws + WS_K + i * D + d4);
    }
    for (int idx = tid; idx < n * CL; idx += 256) {
      const int i = idx / CL, j = idx % CL;
      P_s[i * LDC + j] = ws[WS_P + i * CL + j];
    }
    for (int idx = tid; idx < n * (SLICE / 4); idx += 256) {
      const int i = idx / (SLICE / 4), c4 = (idx % (SLICE / 4)) * 4;
      *reinterpret_cast<float4*>(U_s + i * LDS + c4) = *reinterpret_cast<const float4*>(ws + WS_U + i * D + col0 + c4);
    }
    const float gamma = ws[WS_G];
    __syncthreads();
    // ---- D = U - W S0
    if (oi < n) {
      float acc[8];
#pragma unroll
      for (int x = 0; x < 8; ++x) acc[x] = U_s[oi * LDS + oc + x];
      for (int d = 0; d < D; ++d) {
        const float w = W_s[oi * LDR + d];
        const float4 s0 = *reinterpret_cast<const float4*>(S_s + d * LDS + oc);
        const float4 s1 = *reinterpret_cast<const float4*>(S_s + d * LDS + oc + 4);
        acc[0] -= w * s0.x; acc[1] -= w * s0.y; acc[2] -= w * s0.z; acc[3] -= w * s0.w;
        acc[4] -= w * s1.x; acc[5] -= w * s1.y; acc[6] -= w * s1.z; acc[7] -= w * s1.w;
      }
#pragma unroll
      for (int x = 0; x < 8; ++x) Dl_s[oi * LDS + oc + x] = acc[x];
    }
    __syncthreads();
    // ---- O = (e^G Q) S0 + P D   (pre-norm output of these rows / columns)
    if (oi < n) {
      float acc[8] = {};
      for (int d = 0; d < D; ++d) {
        const float q = Q_s[oi * LDR + d];
        const float4 s0 = *reinterpret_cast<const float4*>(S_s + d * LDS + oc);
        const float4 s1 = *reinterpret_cast<const float4*>(S_s + d * LDS + oc + 4);
        acc[0] += q * s0.x; acc[1] += q * s0.y; acc[2] += q * s0.z; acc[3] += q * s0.w;
        acc[4] += q * s1.x; acc[5] += q * s1.y; acc[6] += q * s1.z; acc[7] += q * s1.w;
      }
      for (int j = 0; j <= oi; ++j) {
        const float p = P_s[oi * LDC + j];
        const float4 d0 = *reinterpret_cast<const float4*>(Dl_s + j * LDS + oc);
        const float4 d1 = *reinterpret_cast<const float4*>(Dl_s + j * LDS + oc + 4);
        acc[0] += p * d0.x; acc[1] += p * d0.y; acc[2] += p * d0.z; acc[3] += p * d0.w;
        acc[4] += p * d1.x; acc[5] += p * d1.y; acc[6] += p * d1.z; acc[7] += p * d1.w;
      }
      float* o = a.o32 + (size_t(t0 + oi) * a.Hv + h) * D + col0 + oc;
      *reinterpret_cast<float4*>(o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(o + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    __syncthreads();
    // ---- S = e^{G_n} S0 + (e^{G_n - G} K)^T D
    {
      float acc[16];
#pragma unroll
      for (int x = 0; x < 16; ++x) acc[x] = gamma * S_s[sd * LDS + sc + x];
      for (int j = 0; j < n; ++j) {
        const float k = K_s[j * LDR + sd];
#pragma unroll
        for (int x = 0; x < 16; x += 4) {
          const float4 dv = *reinterpret_cast<const float4*>(Dl_s + j * LDS + sc + x);
          acc[x] += k * dv.x; acc[x + 1] += k * dv.y; acc[x + 2] += k * dv.z; acc[x + 3] += k * dv.w;
        }
      }
      __syncthreads();
#pragma unroll
      for (int x = 0; x < 16; ++x) S_s[sd * LDS + sc + x] = acc[x];
    }
  }
  __syncthreads();
  for (int idx = tid; idx < D * SLICE; idx += 256) {
    const int d = idx / SLICE, cc = idx % SLICE;
    S[d * D + col0 + cc] = S_s[d * LDS + cc];
  }
  // ---- new conv window (the last KW-1 raw inputs); every prep CTA has finished reading the old one
  if (sv == 0 && c1 > c0) {
    const int r = a.Hv / a.Hk, hk = h / r, kd = a.Hk * D;
    const int seq0 = a.cu_seqlens[s], L = a.cu_seqlens[s + 1] - seq0;
    auto commit = [&](int ch) {
      __nv_bfloat16* cw = a.conv + (size_t(slot) * a.C + ch) * (KW - 1);
      __nv_bfloat16 nv[KW - 1];
#pragma unroll
      for (int i = 0; i < KW - 1; ++i) {
        const int pos = L - (KW - 1) + i;
        nv[i] = pos >= 0 ? a.proj[size_t(seq0 + pos) * a.proj_stride + ch] : cw[(KW - 1) + pos];
      }
#pragma unroll
      for (int i = 0; i < KW - 1; ++i) cw[i] = nv[i];
    };
    if (tid < 128) commit(2 * kd + h * D + tid);               // v channels of this value head
    if (h % r == 0) commit(tid < 128 ? hk * D + tid : kd + hk * D + (tid - 128));  // q / k of the key head
  }
}

// One warp per (token, value head): bf16-rounded output, gated RMSNorm.
__global__ void __launch_bounds__(256) gdn_chunk_norm_kernel(ChunkArgs a) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= a.T * a.Hv) return;
  const int t = row / a.Hv, h = row % a.Hv;
  const float* o = a.o32 + size_t(row) * D;
  float ob[4], ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    ob[e] = __bfloat162float(__float2bfloat16(o[lane + 32 * e]));
    ss += ob[e] * ob[e];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / float(D) + a.eps);
  const __nv_bfloat16* z = a.proj + size_t(t) * a.proj_stride + a.C + h * D;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = lane + 32 * e;
    const float zz = bf(z[d]);
    a.out[size_t(t) * (a.Hv * D) + h * D + d] = __float2bfloat16(ob[e] * inv * bf(a.norm_w[d]) * silu_f(zz));
  }
}

}  // namespace

// chunk_info = [chunk_seq (nc) | chunk_t0 (nc) | chunk_n (nc) | cu_chunks (B+1)] int32 on the device.
at::Tensor gdn_prefill_chunked(const at::Tensor& proj, const at::Tensor& cu_seqlens, const at::Tensor& slots,
                               const at::Tensor& chunk_info, int64_t nc, const at::Tensor& conv_w,
                               const at::Tensor& A_log, const at::Tensor& dt_bias, const at::Tensor& norm_w,
                               at::Tensor rec, at::Tensor conv, int64_t hk, int64_t hv, double eps) {
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && proj.is_contiguous(), "chunked GDN prefill needs bf16 proj");
  TORCH_CHECK(rec.scalar_type() == at::kFloat && rec.is_contiguous() && rec.size(1) == hv && rec.size(2) == D &&
                  rec.size(3) == D, "recurrent pool must be fp32 [S, Hv, 128, 128]");
  TORCH_CHECK(conv.scalar_type() == at::kBFloat16 && conv.is_contiguous() && conv.size(2) == KW - 1, "bad conv pool");
  TORCH_CHECK(hv % hk == 0, "Hv must be a multiple of Hk");
  const int T = proj.size(0), B = slots.numel();
  const int C = conv.size(1);
  TORCH_CHECK(C == (2 * hk + hv) * D, "conv channels must be (2 Hk + Hv) * 128");
  TORCH_CHECK(chunk_info.scalar_type() == at::kInt && chunk_info.numel() == 3 * nc + B + 1, "chunk table size");
  at::Tensor out = at::empty({T, hv * D}, proj.options());
  if (T == 0 || nc == 0) return out;
  at::Tensor ws = at::empty({nc, hv, WS_STRIDE}, proj.options().dtype(at::kFloat));
  at::Tensor o32 = at::empty({T, hv, D}, proj.options().dtype(at::kFloat));
  ChunkArgs a = {};
  a.proj = reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr());
  a.proj_stride = proj.size(1);
  const int* ci = chunk_info.data_ptr<int>();
  a.chunk_seq = ci;
  a.chunk_t0 = ci + nc;
  a.chunk_n = ci + 2 * nc;
  a.cu_chunks = ci + 3 * nc;
  a.cu_seqlens = cu_seqlens.data_ptr<int>();
  a.slots = slots.data_ptr<int>();
  a.conv_w = reinterpret_cast<const __nv_bfloat16*>(conv_w.data_ptr());
  a.A_log = A_log.data_ptr<float>();
  a.dt_bias = dt_bias.data_ptr<float>();
  a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr());
  a.rec = rec.data_ptr<float>();
  a.conv = reinterpret_cast<__nv_bfloat16*>(conv.data_ptr());
  a.ws = ws.data_ptr<float>();
  a.o32 = o32.data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.Hk = hk;
  a.Hv = hv;
  a.C = C;
  a.T = T;
  a.eps = float(eps);
  auto st = at::cuda::getCurrentCUDAStream();
  const int prep_smem = kPrepSmemFloats * 4, state_smem = kStateSmemFloats * 4;
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     prep_smem) == cudaSuccess, "chunk prep smem attribute");
    TORCH_CHECK(cudaFuncSetAttribute(gdn_chunk_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     state_smem) == cudaSuccess, "chunk state smem attribute");
    attr = true;
  }
  launch_pdl(gdn_chunk_prep_kernel, dim3(int(nc), int(hv)), dim3(256), prep_smem, st, a);
  launch_pdl(gdn_chunk_state_kernel, dim3(D / SLICE, int(hv), B), dim3(256), state_smem, st, a);
  launch_pdl(gdn_chunk_norm_kernel, dim3((T * int(hv) + 7) / 8), dim3(256), 0, st, a);
  return out;
}

}  // namespace isb
