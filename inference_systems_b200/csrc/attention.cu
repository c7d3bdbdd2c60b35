// Full-attention kernels over the paged KV cache ([num_blocks, Hkv, 256, hd] bf16 per layer).
//
// attn_prepare:      split the fused projection row (per head: query | gate, then k, v),
//                    per-head RMSNorm of q and k, rotate-half partial RoPE on the
//                    first ``rotary_dim`` channels, write K/V into the cache at
//                    ``slot_mapping`` (replaces the reference's Triton store kernel,
//                    ``nanovllm/layers/attention.py:10-40``, and its torch q/k norm + RoPE).
// attention_decode:  split-KV flash decoding; one CTA per (KV head, sequence, page)
//                    serves the whole GQA group; a combine kernel merges the page
//                    partials and applies the sigmoid output gate.
// attention_prefill: causal varlen attention of the new tokens over all visible
//                    cache rows (prefix-cached rows included), online softmax, GQA
//                    group per CTA, sigmoid output gate fused.

#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <type_traits>

#include "common.cuh"
#include "launch.cuh"

namespace isb {

namespace {

constexpr int PAGE = 256;

__device__ __forceinline__ void load_bf16x8(const __nv_bfloat16* p, float* v) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}


// ------------------------------------------------------------------ prepare
// One warp per (token, head); HD/32 channels per lane (HD in {128, 256}).
template <typename TIn>
__device__ __forceinline__ float take_in(TIn* row, int idx) {
  if constexpr (std::is_same_v<TIn, float>) {
    const float v = row[idx];
    row[idx] = 0.f;  // fp32 accumulator input: its only reader re-zeroes it
    return v;
  } else {
    return __bfloat162float(row[idx]);
  }
}

template <int HD, typename TIn>
__global__ void attn_prepare_kernel(TIn* __restrict__ qkv, int qkv_stride, __nv_bfloat16* __restrict__ gate_out,
                                    const int* __restrict__ pos,
                                    const int* __restrict__ slot_map, const __nv_bfloat16* __restrict__ qn,
                                    const __nv_bfloat16* __restrict__ kn, const float* __restrict__ cos_sin, int rd,
                                    __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                                    __nv_bfloat16* __restrict__ q_out, int T, int Hq, int Hkv, float eps, bool gated,
                                    bool zc) {
  pdl_trigger();
  pdl_wait();
  constexpr int E = HD / 32;
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  const int t = warp_global / heads, hh = warp_global % heads;
  if (t >= T) return;
  TIn* row = qkv + size_t(t) * qkv_stride;
  const int qw = Hq * HD * (gated ? 2 : 1);
  float v[E];
  TIn* src;
  int kind;  // 0 q, 1 k, 2 v
  int head;
  if (hh < Hq) { kind = 0; head = hh; src = row + head * HD * (gated ? 2 : 1); }
  else if (hh < Hq + Hkv) { kind = 1; head = hh - Hq; src = row + qw + head * HD; }
  else { kind = 2; head = hh - Hq - Hkv; src = row + qw + Hkv * HD + head * HD; }
#pragma unroll
  for (int i = 0; i < E; ++i) v[i] = take_in(src, lane * E + i);
  if (kind == 0 && gated) {
    __nv_bfloat16* gdst = gate_out + (size_t(t) * Hq + head) * HD + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) gdst[i] = __float2bfloat16(take_in(src + HD, lane * E + i));
  }
  const int slot = slot_map[t];
  if (kind == 2) {
    if (slot >= 0) {
      const int blk = slot / PAGE, off = slot % PAGE;
      __nv_bfloat16* dst = vc + ((size_t(blk) * Hkv + head) * PAGE + off) * HD + lane * E;
#pragma unroll
      for (int i = 0; i < E; ++i) dst[i] = __float2bfloat16(v[i]);
    }
    return;
  }
  // RMSNorm over the head
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) ss += v[i] * v[i];
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / float(HD) + eps);
  const __nv_bfloat16* w = kind == 0 ? qn : kn;
#pragma unroll
  for (int i = 0; i < E; ++i) {
    const float wi = __bfloat162float(w[lane * E + i]);
    v[i] = zc ? v[i] * rs * (1.f + wi) : __bfloat162float(__float2bfloat16(v[i] * rs)) * wi;
    v[i] = __bfloat162float(__float2bfloat16(v[i]));  // the reference rounds normed q/k to the model dtype
  }
  // rotate-half RoPE on channels [0, rd): pairs (c, c + rd/2)
  const int half = rd / 2;
  const int partner = half / E;  // lane distance between the two halves
  const int p = pos[t];
  float other[E];
#pragma unroll
  for (int i = 0; i < E; ++i) other[i] = __shfl_xor_sync(0xffffffffu, v[i], partner);
  if (lane * E < rd) {
    const bool first = lane * E < half;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const int c = lane * E + i;
      const int f = first ? c : c - half;
      const float cs = cos_sin[size_t(p) * rd + f], sn = cos_sin[size_t(p) * rd + half + f];
      v[i] = first ? v[i] * cs - other[i] * sn : v[i] * cs + other[i] * sn;
    }
  }
  if (kind == 0) {
    __nv_bfloat16* dst = q_out + (size_t(t) * Hq + head) * HD + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) dst[i] = __float2bfloat16(v[i]);
  } else if (slot >= 0) {
    const int blk = slot / PAGE, off = slot % PAGE;
    __nv_bfloat16* dst = kc + ((size_t(blk) * Hkv + head) * PAGE + off) * HD + lane * E;
#pragma unroll
    for (int i = 0; i < E; ++i) dst[i] = __float2bfloat16(v[i]);
  }
}

// ------------------------------------------------------------------ decode
// grid (Hkv, B, chunks of 64 tokens); 256 threads (8 warps).
//   The chunk's K and V rows (contiguous inside a page) are pulled into shared
//   memory with two bulk asynchronous copies completing on one mbarrier, so a
//   CTA keeps 2 x 64 x HD x 2 bytes in flight with no per-thread address math.
//   phase 1: half-warps compute q.k for the whole GQA group (16-lane shuffles;
//            the loop is warp-uniform so every lane reaches every shuffle)
//   phase 2: warp g computes max / exp / sum for head g
//   phase 3: warp w owns HD/8 output channels and accumulates p * v over the chunk
// Partials (o[G][HD], m, l) per (sequence, q head, chunk) are merged by attn_combine_kernel.
constexpr int DCHUNK = 64;

__device__ unsigned int g_attn_err;

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <int HD, int G>
__global__ void __launch_bounds__(256) attn_decode_kernel(const __nv_bfloat16* __restrict__ q,
                                                          const __nv_bfloat16* __restrict__ kc,
                                                          const __nv_bfloat16* __restrict__ vcache,
                                                          const int* __restrict__ ctx_lens,
                                                          const int* __restrict__ block_tables, int max_blocks,
                                                          int Hkv, float scale, float* __restrict__ part_o,
                                                          float* __restrict__ part_ml, int max_chunks) {
  pdl_trigger();
  pdl_wait();
  constexpr int ED = HD / 16;   // channels per lane in phase 1
  constexpr int DW = HD / 8;    // output channels per warp in phase 3
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  __nv_bfloat16* k_s = reinterpret_cast<__nv_bfloat16*>(dsm_raw);   // [64][HD]
  __nv_bfloat16* v_s = k_s + DCHUNK * HD;                            // [64][HD]
  float* q_s = reinterpret_cast<float*>(v_s + DCHUNK * HD);          // [G][HD]
  float* s_s = q_s + G * HD;                                         // [G][64]
  __shared__ uint64_t bar;
  __shared__ float m_s[G], l_s[G];
  const int kvh = blockIdx.x, b = blockIdx.y, chunk = blockIdx.z;
  const int ctx = ctx_lens[b];
  const int start = chunk * DCHUNK;
  const int Hq = Hkv * G;
  const size_t pidx = (size_t(b) * Hq + kvh * G) * max_chunks + chunk;  // + g * max_chunks
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (start >= ctx) {
    if (tid < G) {
      part_ml[(pidx + tid * max_chunks) * 2 + 0] = -INFINITY;
      part_ml[(pidx + tid * max_chunks) * 2 + 1] = 0.f;
    }
    return;
  }
  const int n = min(DCHUNK, ctx - start);
  const int blk = block_tables[b * max_blocks + start / PAGE];
  const size_t row0 = (size_t(blk) * Hkv + kvh) * PAGE + start % PAGE;
  if (tid == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t bytes = uint32_t(n) * HD * 2;
    mbar_arrive_expect_tx(&bar, 2 * bytes);
    bulk_g2s(k_s, kc + row0 * HD, bytes, &bar);
    bulk_g2s(v_s, vcache + row0 * HD, bytes, &bar);
  }
  for (int i = tid; i < G * HD; i += 256) q_s[i] = __bfloat162float(q[(size_t(b) * Hq + kvh * G) * HD + i]) * scale;
  __syncthreads();
  if (!mbar_wait(&bar, 0)) atomicOr(&g_attn_err, 1u);
  // ---- phase 1: scores.  Lane hl of a half-warp owns channels {j*128 + hl*8 .. +8}, so each
  // 16-byte K read of a half-warp covers 256 contiguous bytes (no bank conflicts) and the
  // query slice lives in registers.
  {
    const int hl = lane & 15;
    constexpr int NJ = ED / 8;  // 16-byte chunks per lane
    float qr[G][ED];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) qr[g][j * 8 + e] = q_s[g * HD + j * 128 + hl * 8 + e];
    for (int t0 = warp * 2; t0 < n; t0 += 16) {
      const int t = t0 + (lane >> 4);
      const bool valid = t < n;
      float kv[ED];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        if (valid) {
          const uint4 raw = *reinterpret_cast<const uint4*>(k_s + t * HD + j * 128 + hl * 8);
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h2[e]);
            kv[j * 8 + 2 * e] = f.x;
            kv[j * 8 + 2 * e + 1] = f.y;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) kv[j * 8 + e] = 0.f;
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float sacc = 0.f;
#pragma unroll
        for (int i = 0; i < ED; ++i) sacc += qr[g][i] * kv[i];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, o);
        if (valid && hl == 0) s_s[g * DCHUNK + t] = sacc;
      }
    }
  }
  __syncthreads();
  // ---- phase 2: warp g owns head g (G <= 8)
  if (warp < G) {
    const int g = warp;
    const float a0 = lane < n ? s_s[g * DCHUNK + lane] : -INFINITY;
    const float a1 = lane + 32 < n ? s_s[g * DCHUNK + lane + 32] : -INFINITY;
    const float m = warp_max(fmaxf(a0, a1));
    const float e0 = lane < n ? __expf(a0 - m) : 0.f;
    const float e1 = lane + 32 < n ? __expf(a1 - m) : 0.f;
    s_s[g * DCHUNK + lane] = e0;
    s_s[g * DCHUNK + lane + 32] = e1;
    const float l = warp_sum(e0 + e1);
    if (lane == 0) { m_s[g] = m; l_s[g] = l; }
  }
  __syncthreads();
  // ---- phase 3: P V, warp w owns channels [w*DW, (w+1)*DW)
  if (lane < DW) {
    const int d = warp * DW + lane;
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.f;
    for (int t = 0; t < n; ++t) {
      const float vv = __bfloat162float(v_s[t * HD + d]);
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] += s_s[g * DCHUNK + t] * vv;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) part_o[(pidx + g * max_chunks) * HD + d] = acc[g];
  }
  if (tid < G) {
    part_ml[(pidx + tid * max_chunks) * 2 + 0] = m_s[tid];
    part_ml[(pidx + tid * max_chunks) * 2 + 1] = l_s[tid];
  }
}

// grid (Hq, B); HD threads. Merges chunk partials, applies the output gate.
template <int HD>
__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int max_chunks,
                                    int chunk, const int* __restrict__ ctx_lens, const __nv_bfloat16* __restrict__ gate,
                                    bool gated, __nv_bfloat16* __restrict__ out, int Hq) {
  pdl_trigger();
  pdl_wait();
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int ctx = ctx_lens[b];
  int chunks = (ctx + chunk - 1) / chunk;
  if (chunks > max_chunks) {  // context longer than the block table covers: combine what was computed
    if (d == 0) atomicOr(&g_attn_err, 2u);
    chunks = max_chunks;
  }
  const size_t base = (size_t(b) * Hq + h) * max_chunks;
  float m = -INFINITY;
  for (int p = 0; p < chunks; ++p) m = fmaxf(m, part_ml[(base + p) * 2]);
  float l = 0.f, acc = 0.f;
  for (int p = 0; p < chunks; ++p) {
    const float w = __expf(part_ml[(base + p) * 2] - m);
    l += w * part_ml[(base + p) * 2 + 1];
    acc += w * part_o[(base + p) * HD + d];
  }
  float o = chunks > 0 && l > 0.f ? acc / l : 0.f;
  if (gated) {
    o *= sigmoidf_(__bfloat162float(gate[(size_t(b) * Hq + h) * HD + d]));
  }
  out[(size_t(b) * Hq + h) * HD + d] = __float2bfloat16(o);
}

// ----------------------------------------------------------------- prefill
// grid (q_tiles, Hkv, B); 256 threads; QT queries x G heads per CTA, key tiles of KT.
template <int HD, int G, int QT>
__global__ void __launch_bounds__(256) attn_prefill_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc, const __nv_bfloat16* __restrict__ vcache,
    const int* __restrict__ cu_q, const int* __restrict__ ctx_lens, const int* __restrict__ block_tables,
    int max_blocks, int Hkv, float scale, const __nv_bfloat16* __restrict__ gate, bool gated,
    __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  constexpr int R = QT * G;        // query rows (query-major, head-minor)
  constexpr int KT = 32;           // keys per tile
  extern __shared__ float sm[];
  float* q_s = sm;                          // [R][HD]
  float* k_s = q_s + R * HD;                // [KT][HD + 1]
  float* v_s = k_s + KT * (HD + 1);         // [KT][HD]
  float* s_s = v_s + KT * HD;               // [R][KT]
  float* m_s = s_s + R * KT;                // [R]
  float* l_s = m_s + R;                     // [R]
  float* a_s = l_s + R;                     // [R] rescale factors
  const int qt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int q0 = cu_q[b], nq = cu_q[b + 1] - q0;
  const int tq0 = qt * QT;
  if (tq0 >= nq) return;
  const int ctx = ctx_lens[b];
  const int past = ctx - nq;          // cached tokens before the first new query
  const int Hq = Hkv * G;
  const int tid = threadIdx.x;
  const int nrows = min(QT, nq - tq0) * G;
  for (int i = tid; i < R * HD; i += 256) {
    const int r = i / HD, d = i % HD;
    const int qi = r / G, g = r % G;
    float val = 0.f;
    if (qi < min(QT, nq - tq0)) val = __bfloat162float(q[(size_t(q0 + tq0 + qi) * Hq + kvh * G + g) * HD + d]) * scale;
    q_s[i] = val;
  }
  for (int r = tid; r < R; r += 256) { m_s[r] = -INFINITY; l_s[r] = 0.f; }
  // each thread owns output rows/channels: R*HD / 256 accumulators
  constexpr int PER = R * HD / 256;
  float acc[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) acc[i] = 0.f;
  const int last_q_pos = past + min(QT, nq - tq0) - 1 + tq0;
  const int kend = last_q_pos + 1;  // keys [0, kend)
  __syncthreads();
  for (int k0 = 0; k0 < kend; k0 += KT) {
    const int nk = min(KT, kend - k0);
    for (int i = tid; i < KT * HD; i += 256) {
      const int kk = i / HD, d = i % HD;
      float kvv = 0.f, vvv = 0.f;
      if (kk < nk) {
        const int pos = k0 + kk;
        const int blk = block_tables[b * max_blocks + pos / PAGE];
        const size_t off = ((size_t(blk) * Hkv + kvh) * PAGE + pos % PAGE) * HD + d;
        kvv = __bfloat162float(kc[off]);
        vvv = __bfloat162float(vcache[off]);
      }
      k_s[kk * (HD + 1) + d] = kvv;
      v_s[kk * HD + d] = vvv;
    }
    __syncthreads();
    // scores R x KT
    for (int i = tid; i < R * KT; i += 256) {
      const int r = i / KT, kk = i % KT;
      const int qpos = past + tq0 + r / G;
      float s = -INFINITY;
      if (r < nrows && kk < nk && k0 + kk <= qpos) {
        s = 0.f;
        const float* qr = q_s + r * HD;
        const float* kr = k_s + kk * (HD + 1);
#pragma unroll 8
        for (int d = 0; d < HD; ++d) s += qr[d] * kr[d];
      }
      s_s[i] = s;
    }
    __syncthreads();
    // online softmax per row
    for (int r = tid; r < R; r += 256) {
      float mx = m_s[r];
      for (int kk = 0; kk < KT; ++kk) mx = fmaxf(mx, s_s[r * KT + kk]);
      float l = 0.f;
      for (int kk = 0; kk < KT; ++kk) {
        const float e = mx == -INFINITY ? 0.f : __expf(s_s[r * KT + kk] - mx);
        s_s[r * KT + kk] = e;
        l += e;
      }
      const float alpha = m_s[r] == -INFINITY ? 0.f : __expf(m_s[r] - mx);
      a_s[r] = alpha;
      l_s[r] = l_s[r] * alpha + l;
      m_s[r] = mx;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = tid + i * 256;
      const int r = idx / HD, d = idx % HD;
      float a = acc[i] * a_s[r];
      for (int kk = 0; kk < nk; ++kk) a += s_s[r * KT + kk] * v_s[kk * HD + d];
      acc[i] = a;
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int idx = tid + i * 256;
    const int r = idx / HD, d = idx % HD;
    if (r >= nrows) continue;
    const int qi = r / G, g = r % G;
    const int t = q0 + tq0 + qi;
    const int h = kvh * G + g;
    float o = l_s[r] > 0.f ? acc[i] / l_s[r] : 0.f;
    if (gated) o *= sigmoidf_(__bfloat162float(gate[(size_t(t) * Hq + h) * HD + d]));
    out[(size_t(t) * Hq + h) * HD + d] = __float2bfloat16(o);
  }
}

void check_cache(const at::Tensor& kc, const at::Tensor& vc, int64_t hd) {
  TORCH_CHECK(kc.dim() == 4 && kc.size(2) == PAGE && kc.size(3) == hd, "KV cache must be [blocks, Hkv, 256, hd]");
  TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous() && kc.scalar_type() == at::kBFloat16, "KV cache layout");
}

}  // namespace

std::tuple<at::Tensor, at::Tensor> attn_prepare(const at::Tensor& qkv, const at::Tensor& positions,
                                                const at::Tensor& slot_mapping, const at::Tensor& qn,
                                                const at::Tensor& kn, const at::Tensor& cos_sin, at::Tensor kc,
                                                at::Tensor vc, int64_t Hq, int64_t Hkv, int64_t hd, double eps,
                                                bool gated, bool zc) {
  check_cache(kc, vc, hd);
  TORCH_CHECK(qkv.is_contiguous() && (qkv.scalar_type() == at::kBFloat16 || qkv.scalar_type() == at::kFloat),
              "qkv must be contiguous bf16 (or an fp32 accumulator, consumed)");
  TORCH_CHECK(positions.scalar_type() == at::kInt && slot_mapping.scalar_type() == at::kInt, "int32 metadata");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "cos/sin table must be fp32");
  const int T = positions.numel();
  const int rd = cos_sin.size(1);
  at::Tensor q = at::empty({T, Hq, hd}, kc.options());
  at::Tensor gate = at::empty({gated ? T : 0, Hq * hd}, kc.options());
  if (T == 0) return {q, gate};
  TORCH_CHECK((rd / 2) % (hd / 32) == 0 && rd <= hd, "rotary dim must split evenly across lanes");
  const int partner = (rd / 2) / (hd / 32);
  TORCH_CHECK(partner > 0 && (partner & (partner - 1)) == 0, "rotary half must map to a power-of-two lane distance");
  const int warps = T * (Hq + 2 * Hkv);
  const int threads = 256;
  const int blocks = (warps * 32 + threads - 1) / threads;
  auto st = at::cuda::getCurrentCUDAStream();
#define ISB_PREP(HD_, T_)                                                                                         \
  launch_pdl(attn_prepare_kernel<HD_, T_>, dim3(blocks), dim3(threads), 0, st,                                                        \
      reinterpret_cast<T_*>(qkv.data_ptr()), qkv.size(1), reinterpret_cast<__nv_bfloat16*>(gate.data_ptr()),      \
      positions.data_ptr<int>(), slot_mapping.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(qn.data_ptr()), \
      reinterpret_cast<const __nv_bfloat16*>(kn.data_ptr()), cos_sin.data_ptr<float>(), rd,                       \
      reinterpret_cast<__nv_bfloat16*>(kc.data_ptr()), reinterpret_cast<__nv_bfloat16*>(vc.data_ptr()),          \
      reinterpret_cast<__nv_bfloat16*>(q.data_ptr()), T, Hq, Hkv, float(eps), gated, zc)
  const bool f32 = qkv.scalar_type() == at::kFloat;
  if (hd == 256) { if (f32) ISB_PREP(256, float); else ISB_PREP(256, __nv_bfloat16); }
  else if (hd == 128) { if (f32) ISB_PREP(128, float); else ISB_PREP(128, __nv_bfloat16); }
  else TORCH_CHECK(false, "attn_prepare supports head_dim 128 or 256");
#undef ISB_PREP
  return {q, gate};
}

bool attention_decode_tc_supported(int64_t hd, int64_t hq, int64_t hkv);
void attention_decode_tc_partials(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc,
                                  const at::Tensor& ctx_lens, const at::Tensor& block_tables, double scale,
                                  at::Tensor& part_o, at::Tensor& part_ml, int max_chunks);

// ISB_ATTN_DECODE_TC: 0 = split-KV SIMT kernel only, 1 = tensor-core kernel whenever the head
// layout allows, unset = tensor cores from 16 (sequence, KV head) pairs up.
int attn_decode_tc_mode() {
  static const int mode = [] {
    const char* e = std::getenv("ISB_ATTN_DECODE_TC");
    return e ? std::atoi(e) : 2;
  }();
  return mode;
}

// Tensor-core split-KV decode (128-key chunks) followed by the combine kernel.
at::Tensor attention_decode_tc(const at::Tensor& q, const at::Tensor& gate, const at::Tensor& kc, const at::Tensor& vc,
                               const at::Tensor& ctx_lens, const at::Tensor& block_tables, double scale, bool gated) {
  const int B = q.size(0), Hq = q.size(1), hd = q.size(2);
  check_cache(kc, vc, hd);
  TORCH_CHECK(ctx_lens.scalar_type() == at::kInt && block_tables.scalar_type() == at::kInt, "int32 metadata");
  at::Tensor out = at::empty({B, Hq * hd}, q.options());
  if (B == 0) return out;
  constexpr int TCHUNK = 128;
  const int max_chunks = block_tables.size(1) * (PAGE / TCHUNK);
  at::Tensor part_o = at::empty({B, Hq, max_chunks, hd}, q.options().dtype(at::kFloat));
  at::Tensor part_ml = at::empty({B, Hq, max_chunks, 2}, q.options().dtype(at::kFloat));
  attention_decode_tc_partials(q, kc, vc, ctx_lens, block_tables, scale, part_o, part_ml, max_chunks);
  launch_pdl(attn_combine_kernel<256>, dim3(Hq, B), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             part_o.data_ptr<float>(), part_ml.data_ptr<float>(), max_chunks, TCHUNK, ctx_lens.data_ptr<int>(),
             reinterpret_cast<const __nv_bfloat16*>(gate.data_ptr()), gated,
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), Hq);
  return out;
}

at::Tensor attention_decode(const at::Tensor& q, const at::Tensor& gate, const at::Tensor& kc, const at::Tensor& vc,
                            const at::Tensor& ctx_lens, const at::Tensor& block_tables, double scale, bool gated) {
  const int B = q.size(0), Hq = q.size(1), hd = q.size(2);
  check_cache(kc, vc, hd);
  TORCH_CHECK(q.is_contiguous() && q.scalar_type() == at::kBFloat16, "q must be contiguous bf16");
  TORCH_CHECK(ctx_lens.scalar_type() == at::kInt && block_tables.scalar_type() == at::kInt, "int32 metadata");
  const int Hkv = kc.size(1);
  const int G = Hq / Hkv;
  const int max_blocks = block_tables.size(1);
  const int tc_mode = attn_decode_tc_mode();
  if (tc_mode != 0 && attention_decode_tc_supported(hd, Hq, Hkv) && (tc_mode == 1 || B * Hkv >= 16))
    return attention_decode_tc(q, gate, kc, vc, ctx_lens, block_tables, scale, gated);
  at::Tensor out = at::empty({B, Hq * hd}, q.options());
  if (B == 0) return out;
  const int max_chunks = max_blocks * (PAGE / DCHUNK);
  at::Tensor part_o = at::empty({B, Hq, max_chunks, hd}, q.options().dtype(at::kFloat));
  at::Tensor part_ml = at::empty({B, Hq, max_chunks, 2}, q.options().dtype(at::kFloat));
  auto st = at::cuda::getCurrentCUDAStream();
  const dim3 grid(Hkv, B, max_chunks);
  bool launched = false;
  auto launch = [&](auto hd_c, auto g_c) {
    constexpr int HD_ = decltype(hd_c)::value, G_ = decltype(g_c)::value;
    if (hd != HD_ || G != G_ || launched) return;
    const int smem = 2 * DCHUNK * HD_ * 2 + (G_ * HD_ + G_ * DCHUNK) * 4;
    auto kern = attn_decode_kernel<HD_, G_>;
    static bool attr = false;
    if (!attr) {
      TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess);
      attr = true;
    }
    launch_pdl(kern, dim3(grid), dim3(256), smem, st, reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()),
                                  reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr()),
                                  reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr()), ctx_lens.data_ptr<int>(),
                                  block_tables.data_ptr<int>(), max_blocks, Hkv, float(scale),
                                  part_o.data_ptr<float>(), part_ml.data_ptr<float>(), max_chunks);
    launched = true;
  };
#define ISB_DEC_G(HD_, G_) launch(std::integral_constant<int, HD_>{}, std::integral_constant<int, G_>{});
  ISB_DEC_G(256, 1) ISB_DEC_G(256, 2) ISB_DEC_G(256, 3) ISB_DEC_G(256, 4) ISB_DEC_G(256, 6) ISB_DEC_G(256, 8)
  ISB_DEC_G(128, 1) ISB_DEC_G(128, 2) ISB_DEC_G(128, 4)
#undef ISB_DEC_G
  TORCH_CHECK(launched, "attention_decode: unsupported (head_dim, group) = (", hd, ", ", G, ")");
#define ISB_COMB(HD_)                                                                                              \
  launch_pdl(attn_combine_kernel<HD_>, dim3(dim3(Hq, B)), dim3(HD_), 0, st, part_o.data_ptr<float>(), part_ml.data_ptr<float>(),       \
                                                       max_chunks, DCHUNK, ctx_lens.data_ptr<int>(),                  \
                                                       reinterpret_cast<const __nv_bfloat16*>(gate.data_ptr()),      \
                                                       gated,                                                        \
                                                       reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), Hq)
  if (hd == 256) ISB_COMB(256); else ISB_COMB(128);
#undef ISB_COMB
  return out;
}

int64_t attn_error_word() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_attn_err, sizeof(v));
  const unsigned int z = 0;
  cudaMemcpyToSymbol(g_attn_err, &z, sizeof(z));
  return v;
}

// Device address of the error word (read by the per-step status kernel).
int64_t attn_error_word_address() {
  void* p = nullptr;
  TORCH_CHECK(cudaGetSymbolAddress(&p, g_attn_err) == cudaSuccess, "error word address");
  return reinterpret_cast<int64_t>(p);
}

at::Tensor attention_prefill(const at::Tensor& q, const at::Tensor& gate, const at::Tensor& kc, const at::Tensor& vc,
                             const at::Tensor& cu_q, const at::Tensor& ctx_lens, const at::Tensor& block_tables,
                             double scale, bool gated, int64_t max_seqlen_q) {
  const int T = q.size(0), Hq = q.size(1), hd = q.size(2);
  check_cache(kc, vc, hd);
  const int Hkv = kc.size(1);
  const int G = Hq / Hkv;
  const int B = ctx_lens.numel();
  at::Tensor out = at::empty({T, Hq * hd}, q.options());
  if (T == 0) return out;
  auto st = at::cuda::getCurrentCUDAStream();
#define ISB_PRE(HD_, G_, QT_)                                                                                       \
  do {                                                                                                             \
    constexpr int R = QT_ * G_;                                                                                   \
    const int smem = (R * HD_ + 32 * (HD_ + 1) + 32 * HD_ + R * 32 + 3 * R) * 4;                                  \
    auto kern = attn_prefill_kernel<HD_, G_, QT_>;                                                                 \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);                                \
    const dim3 grid((max_seqlen_q + QT_ - 1) / QT_, Hkv, B);                                                       \
    launch_pdl(kern, dim3(grid), dim3(256), smem, st, reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()),                           \
                                  reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr()),                          \
                                  reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr()), cu_q.data_ptr<int>(),    \
                                  ctx_lens.data_ptr<int>(), block_tables.data_ptr<int>(), block_tables.size(1),    \
                                  Hkv, float(scale), reinterpret_cast<const __nv_bfloat16*>(gate.data_ptr()),     \
                                  gated, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));                       \
  } while (0)
  if (hd == 256 && G == 4) ISB_PRE(256, 4, 16);
  else if (hd == 256 && G == 2) ISB_PRE(256, 2, 32);
  else if (hd == 256 && G == 6) ISB_PRE(256, 6, 8);
  else if (hd == 256 && G == 3) ISB_PRE(256, 3, 16);
  else if (hd == 256 && G == 8) ISB_PRE(256, 8, 8);
  else if (hd == 256 && G == 1) ISB_PRE(256, 1, 32);
  else if (hd == 128 && G == 2) ISB_PRE(128, 2, 32);
  else if (hd == 128 && G == 1) ISB_PRE(128, 1, 64);
  else if (hd == 128 && G == 4) ISB_PRE(128, 4, 16);
  else TORCH_CHECK(false, "attention_prefill: unsupported (head_dim, group) = (", hd, ", ", G, ")");
#undef ISB_PRE
  return out;
}

}  // namespace isb

// ------------------------------------------------------------ no-alloc entry
// The C entry point declared in noalloc.h (no counterpart in the reference):
// the same decode + combine kernels as attention_decode, with the split-KV
// partials in a fixed device array instead of tensors from the allocator.
#include <mutex>

#include "noalloc.h"

namespace isb {
namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[ISB_NOALLOC_SCRATCH_BYTES];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[kNoAllocMaxDevices] = {};

size_t part_o_bytes(int B, int Hq, int hd, int max_chunks) {
  return (size_t(B) * Hq * max_chunks * hd * sizeof(float) + 255) / 256 * 256;
}

template <int HD, int G>
int decode_smem() {
  return 2 * DCHUNK * HD * 2 + (G * HD + G * DCHUNK) * 4;
}

template <int HD, int G>
bool set_decode_attr() {
  return cudaFuncSetAttribute(attn_decode_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              decode_smem<HD, G>()) == cudaSuccess;
}

// Returns this device's scratch pointer, running the one-time set-up first.
unsigned char* noalloc_scratch(int* code) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    *code = ISB_NOALLOC_ESETUP;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      *code = ISB_NOALLOC_ESETUP;
      return nullptr;
    }
    const bool ok = set_decode_attr<256, 1>() && set_decode_attr<256, 2>() && set_decode_attr<256, 3>() &&
                    set_decode_attr<256, 4>() && set_decode_attr<256, 6>() && set_decode_attr<256, 8>() &&
                    set_decode_attr<128, 1>() && set_decode_attr<128, 2>() && set_decode_attr<128, 4>();
    if (!ok) {
      *code = ISB_NOALLOC_ESETUP;
      return nullptr;
    }
    g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *code = ISB_NOALLOC_OK;
  return g_noalloc_ptr[dev];
}

template <int HD, int G>
void launch_decode_noalloc(const __nv_bfloat16* q, const __nv_bfloat16* kc, const __nv_bfloat16* vc,
                           const int* ctx_lens, const int* bt, int max_blocks, int B, int Hkv, float scale,
                           float* part_o, float* part_ml, int max_chunks, cudaStream_t st) {
  attn_decode_kernel<HD, G><<<dim3(Hkv, B, max_chunks), 256, decode_smem<HD, G>(), st>>>(
      q, kc, vc, ctx_lens, bt, max_blocks, Hkv, scale, part_o, part_ml, max_chunks);
}

}  // namespace
}  // namespace isb

extern "C" {

__attribute__((visibility("default"))) size_t isb_attention_decode_noalloc_scratch_bytes(int batch, int num_q_heads,
                                                                                         int head_dim,
                                                                                         int max_blocks) {
  if (batch <= 0 || num_q_heads <= 0 || head_dim <= 0 || max_blocks <= 0) return 0;
  const size_t max_chunks = size_t(max_blocks) * (isb::PAGE / isb::DCHUNK);  // size_t: no int overflow
  const size_t part_o = (size_t(batch) * num_q_heads * max_chunks * head_dim * sizeof(float) + 255) / 256 * 256;
  return part_o + size_t(batch) * num_q_heads * max_chunks * 2 * sizeof(float);
}

__attribute__((visibility("default"))) int isb_noalloc_setup(void) {
  int code = ISB_NOALLOC_OK;
  isb::noalloc_scratch(&code);
  return code;
}

__attribute__((visibility("default"))) int isb_attention_decode_noalloc(
    const void* q, const void* gate, const void* k_cache, const void* v_cache, const int* ctx_lens,
    const int* block_tables, int max_blocks, int batch, int num_q_heads, int num_kv_heads, int head_dim, float scale,
    void* out, cudaStream_t stream) {
  if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_blocks <= 0)
    return ISB_NOALLOC_EINVAL;
  // The decode grid has one z-slice per 64-token chunk and gridDim.z stops at 65535.
  if (max_blocks > ISB_NOALLOC_MAX_BLOCKS || batch > 65535) return ISB_NOALLOC_EINVAL;
  // Size check first: it never touches a pointer.
  const size_t need = isb_attention_decode_noalloc_scratch_bytes(batch, num_q_heads, head_dim, max_blocks);
  if (need > ISB_NOALLOC_SCRATCH_BYTES) return ISB_NOALLOC_ETOOBIG;
  if (!q || !k_cache || !v_cache || !ctx_lens || !block_tables || !out) return ISB_NOALLOC_EINVAL;
  if (num_q_heads % num_kv_heads != 0) return ISB_NOALLOC_EUNSUPPORTED;
  const int G = num_q_heads / num_kv_heads;
  const bool hd256 = head_dim == 256 && (G == 1 || G == 2 || G == 3 || G == 4 || G == 6 || G == 8);
  const bool hd128 = head_dim == 128 && (G == 1 || G == 2 || G == 4);
  if (!hd256 && !hd128) return ISB_NOALLOC_EUNSUPPORTED;

  // An error left pending by earlier work of the caller stays theirs: report it without clearing it
  // and launch nothing, so the check after the launches below covers only this call's kernels.
  if (cudaPeekAtLastError() != cudaSuccess) return ISB_NOALLOC_EPENDING;
  int code = ISB_NOALLOC_OK;
  unsigned char* scratch = isb::noalloc_scratch(&code);
  if (scratch == nullptr) return code;
  const int max_chunks = max_blocks * (isb::PAGE / isb::DCHUNK);
  float* part_o = reinterpret_cast<float*>(scratch);
  float* part_ml = reinterpret_cast<float*>(scratch + isb::part_o_bytes(batch, num_q_heads, head_dim, max_chunks));

  const auto* qb = static_cast<const __nv_bfloat16*>(q);
  const auto* kb = static_cast<const __nv_bfloat16*>(k_cache);
  const auto* vb = static_cast<const __nv_bfloat16*>(v_cache);
#define ISB_NA_DEC(HD_, G_)                                                                                   \
  if (head_dim == HD_ && G == G_)                                                                             \
    isb::launch_decode_noalloc<HD_, G_>(qb, kb, vb, ctx_lens, block_tables, max_blocks, batch, num_kv_heads,   \
                                        scale, part_o, part_ml, max_chunks, stream);
  ISB_NA_DEC(256, 1) ISB_NA_DEC(256, 2) ISB_NA_DEC(256, 3) ISB_NA_DEC(256, 4) ISB_NA_DEC(256, 6) ISB_NA_DEC(256, 8)
  ISB_NA_DEC(128, 1) ISB_NA_DEC(128, 2) ISB_NA_DEC(128, 4)
#undef ISB_NA_DEC
  const auto* gb = static_cast<const __nv_bfloat16*>(gate);
  auto* ob = static_cast<__nv_bfloat16*>(out);
  if (head_dim == 256)
    isb::attn_combine_kernel<256><<<dim3(num_q_heads, batch), 256, 0, stream>>>(
        part_o, part_ml, max_chunks, isb::DCHUNK, ctx_lens, gb, gb != nullptr, ob, num_q_heads);
  else
    isb::attn_combine_kernel<128><<<dim3(num_q_heads, batch), 128, 0, stream>>>(
        part_o, part_ml, max_chunks, isb::DCHUNK, ctx_lens, gb, gb != nullptr, ob, num_q_heads);
  return cudaGetLastError() == cudaSuccess ? ISB_NOALLOC_OK : ISB_NOALLOC_ELAUNCH;
}

__attribute__((visibility("default"))) unsigned int isb_noalloc_error_word(void) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, isb::g_attn_err, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  const unsigned int z = 0;
  cudaMemcpyToSymbol(isb::g_attn_err, &z, sizeof(z));
  return v;
}

__attribute__((visibility("default"))) const char* isb_noalloc_strerror(int code) {
  switch (code) {
    case ISB_NOALLOC_OK: return "ok";
    case ISB_NOALLOC_ETOOBIG: return "split-KV partials exceed the fixed scratch array (ISB_NOALLOC_SCRATCH_BYTES)";
    case ISB_NOALLOC_EUNSUPPORTED: return "unsupported (head_dim, q heads per kv head)";
    case ISB_NOALLOC_EINVAL: return "null pointer or non-positive size";
    case ISB_NOALLOC_ESETUP: return "per-device set-up failed (cudaGetSymbolAddress or kernel attribute)";
    case ISB_NOALLOC_ELAUNCH: return "kernel launch failed";
    case ISB_NOALLOC_EPENDING: return "a CUDA error from earlier work was pending; nothing was launched";
    default: return "unknown code";
  }
}

}  // extern "C"
