// Gated DeltaNet (GDN) kernels, fp32 recurrent state updated IN PLACE in the slot pool.
//
// gdn_scan: one CTA per (key head, sequence) runs the whole mixer core for the
//   key head's group of value heads:
//     causal depthwise conv (width 4) over q|k|v channels with the conv-state
//     window in registers -> SiLU -> L2-normalise q, k (q * 1/sqrt(Dk)) ->
//     beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) ->
//     S <- e^g S;  delta = (v - k^T S) beta;  S <- S + k delta^T;  o = q^T S ->
//     gated RMSNorm: norm(bf16(o)) * w * SiLU(z)
//   (math: ``nanovllm/models/qwen35_reference.py:52-386``; the reference's CUDA
//   decode kernel ``nanovllm/csrc/gdn_decode_kernel.cu`` handles only Hk == Hv and
//   copies states through gather/scatter; here Hv = r * Hk and the pools are
//   addressed by slot id).
//   Each thread owns a 16 x 4 register tile of the 128 x 128 state (rows
//   16*kr .. +15, columns 4*lane .. +3), so k^T S and q^T S are formed in one
//   pass over the state and the state is read and written exactly once per
//   sequence (decode: once per token).  One CTA per key head makes the
//   shared q/k conv-state update race-free when Hv > Hk.
//   Optional outputs: per-token state history (MTP verify / prefix
//   checkpoints) and compact replay records (k, delta, g).
// gdn_replay_commit: fold accepted (k, delta, g) records into the pool.
// gdn_conv_commit:   copy an accepted conv window from a history into the pool.

#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <type_traits>

#include "common.cuh"
#include "launch.cuh"

namespace isb {

namespace {

constexpr int D = 128;          // key == value head dim handled by these kernels
constexpr int KW = 4;           // conv width
constexpr int kThreads = 256;   // 8 row groups x 32 column groups

__device__ unsigned int g_gdn_err;

// One bulk asynchronous copy of a 64 KB state (global -> this CTA's shared memory), completing
// on ``bar``.  Plain copy: no cluster multicast.
__device__ __forceinline__ void bulk_g2s_state(float* dst, const float* src, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(uint32_t(D * D * 4)), "r"(smem_u32(bar))
               : "memory");
}

struct ScanArgs {
  const void* proj;        // [T, proj_stride] bf16, or fp32 accumulator that is consumed (read, then zeroed)
  int proj_stride;
  const int* cu_seqlens;   // [B+1] or nullptr (one token per sequence)
  const int* slots;        // [B]
  const __nv_bfloat16* conv_w;  // [C, 4]
  const float* A_log;
  const float* dt_bias;
  const __nv_bfloat16* norm_w;  // [D]
  float* rec;              // [S, Hv, D, D]
  __nv_bfloat16* conv;     // [S, C, 3]
  __nv_bfloat16* out;      // [T, Hv*D]
  int Hk, Hv, C;
  float eps;
  bool write_final;        // write the final state back to the pool
  const int* hist_row;     // [T] history row per token (-1: none) or nullptr
  float* hist_rec;         // [rows, Hv, D, D]
  __nv_bfloat16* hist_conv;  // [rows, C, 3]
  float* rec_k;            // [T, Hv, D] replay records or nullptr
  float* rec_delta;        // [T, Hv, D]
  float* rec_g;            // [T, Hv]
};

__device__ __forceinline__ float softplusf(float x) { return x > 20.f ? x : log1pf(expf(x)); }

__device__ __forceinline__ float block_sum_128(float v, float* scratch, int tid) {
  // sum over threads 0..127 (4 warps); every caller thread participates in the syncs
  v = warp_sum(v);
  if ((tid & 31) == 0 && tid < 128) scratch[tid >> 5] = v;
  __syncthreads();
  const float r = scratch[0] + scratch[1] + scratch[2] + scratch[3];
  __syncthreads();
  return r;
}

template <typename TIn>
__device__ __forceinline__ float take(const TIn* row, int idx, bool consume) {
  if constexpr (std::is_same_v<TIn, float>) {
    float* p = const_cast<float*>(row) + idx;
    const float v = *p;
    if (consume) *p = 0.f;
    return v;
  } else {
    return __bfloat162float(row[idx]);
  }
}

// PERSIST (decode only): a grid of about two CTAs per SM walks the (key head, sequence) items;
// each value head's 64 KB state is fetched into shared memory by one bulk asynchronous copy,
// and the next one is requested as soon as every thread has the current state in registers,
// so the state stream overlaps the per-token math and the write-back of the previous state.
template <typename TIn, bool PERSIST>
__global__ void __launch_bounds__(kThreads) gdn_scan_kernel(ScanArgs a, int nitems) {
  pdl_trigger();
  // Nothing is read before the wait: the state pools are also written by plainly launched
  // kernels (slot zeroing on allocation, checkpoint restore, MTP commit), and a dependent
  // launch may start before such a kernel's writes are visible.
  pdl_wait();
  __shared__ float q_s[D], k_s[D], v_s[D], d_s[D];
  __shared__ float red_k[8][D], red_q[8][D];
  __shared__ float scal[16];
  __shared__ float nrm[8], ep[4];
  __shared__ __align__(8) uint64_t st_bar;
  extern __shared__ __align__(128) float st_s[];  // [D][D] prefetched state (PERSIST)

  const int tid = threadIdx.x;
  const int kr = tid >> 5, vc = (tid & 31) * 4;
  const int r = a.Hv / a.Hk;
  // item order: (sequence, key head); value head j of an item is state unit (item * r + j)
  auto unit_src = [&](int unit) -> const float* {
    const int it = unit / r, jj = unit % r;
    const int bb = it / a.Hk, hh = (it % a.Hk) * r + jj;
    return a.rec + ((size_t(a.slots[bb]) * a.Hv + hh) * D) * D;
  };
  auto issue_state = [&](int u) {  // bulk copy of state unit ``u`` into shared memory
    mbar_arrive_expect_tx(&st_bar, D * D * 4);
    bulk_g2s_state(st_s, unit_src(u), &st_bar);
  };
  uint32_t st_phase = 0;
  int unit = PERSIST ? int(blockIdx.x) * r : 0;
  if constexpr (PERSIST) {
    if (tid == 0) {
      mbar_init(&st_bar, 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0 && int(blockIdx.x) < nitems) issue_state(unit);
  }
  for (int item = PERSIST ? int(blockIdx.x) : 0; PERSIST ? item < nitems : item < 1;
       item += PERSIST ? int(gridDim.x) : 1) {
  const int hk = PERSIST ? item % a.Hk : blockIdx.x, b = PERSIST ? item / a.Hk : blockIdx.y;
  const int t0 = a.cu_seqlens ? a.cu_seqlens[b] : b;
  const int t1 = a.cu_seqlens ? a.cu_seqlens[b + 1] : b + 1;
  const int slot = a.slots[b];
  const int kd = a.Hk * D;
  // q/k channel of this thread (threads 0..127: q, 128..255: k)
  const int qk_ch = tid < 128 ? hk * D + tid : kd + hk * D + (tid - 128);
  const float wq0 = __bfloat162float(a.conv_w[qk_ch * KW + 0]), wq1 = __bfloat162float(a.conv_w[qk_ch * KW + 1]),
              wq2 = __bfloat162float(a.conv_w[qk_ch * KW + 2]), wq3 = __bfloat162float(a.conv_w[qk_ch * KW + 3]);
  const float inv_sqrt_d = rsqrtf(float(D));

  for (int j = 0; j < r; ++j) {
    const int h = hk * r + j;
    // conv windows (registers); the pool is not modified until the end
    __nv_bfloat16* cq = a.conv + (size_t(slot) * a.C + qk_ch) * (KW - 1);
    float qs0 = __bfloat162float(cq[0]), qs1 = __bfloat162float(cq[1]), qs2 = __bfloat162float(cq[2]);
    const int v_ch = 2 * kd + h * D + (tid & 127);
    float vs0 = 0.f, vs1 = 0.f, vs2 = 0.f, wv0 = 0.f, wv1 = 0.f, wv2 = 0.f, wv3 = 0.f;
    if (tid < 128) {
      const __nv_bfloat16* cv = a.conv + (size_t(slot) * a.C + v_ch) * (KW - 1);
      vs0 = __bfloat162float(cv[0]); vs1 = __bfloat162float(cv[1]); vs2 = __bfloat162float(cv[2]);
      wv0 = __bfloat162float(a.conv_w[v_ch * KW + 0]); wv1 = __bfloat162float(a.conv_w[v_ch * KW + 1]);
      wv2 = __bfloat162float(a.conv_w[v_ch * KW + 2]); wv3 = __bfloat162float(a.conv_w[v_ch * KW + 3]);
    }
    const float A = -expf(a.A_log[h]);
    const float dtb = a.dt_bias[h];
    // state tile
    float* S = a.rec + ((size_t(slot) * a.Hv + h) * D) * D;
    float4 st[16];
    if constexpr (PERSIST) {
      if (!mbar_wait(&st_bar, st_phase)) atomicOr(&g_gdn_err, 1u);
      st_phase ^= 1u;
#pragma unroll
      for (int i = 0; i < 16; ++i) st[i] = *reinterpret_cast<const float4*>(st_s + (kr * 16 + i) * D + vc);
      __syncthreads();  // every thread holds its part of the state: the buffer is free
      unit = (j + 1 < r) ? unit + 1 : (item + int(gridDim.x)) * r;
      if (tid == 0 && unit / r < nitems) issue_state(unit);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) st[i] = *reinterpret_cast<const float4*>(S + (kr * 16 + i) * D + vc);
    }

    // Four block barriers per token.  q and k stay unnormalised in shared memory: their L2
    // norms are reduced together with the k^T S / q^T S partial sums and applied as scalars
    // (k^T S, q^T S, q.k and the key of the state update all scale linearly).
    for (int t = t0; t < t1; ++t) {
      const TIn* x = static_cast<const TIn*>(a.proj) + size_t(t) * a.proj_stride;
      // --- every input of this token first (an fp32 accumulator input is re-zeroed by its only reader)
      const float xq = take(x, qk_ch, j == r - 1);
      float xv = 0.f, z = 0.f;
      if (tid < 128) {
        xv = take(x, v_ch, true);
        z = take(x, a.C + h * D + tid, true);
      }
      float bb = 0.f, aa = 0.f;
      if (tid == 0) {
        bb = take(x, a.C + a.Hv * D + h, true);
        aa = take(x, a.C + a.Hv * D + a.Hv + h, true);
      }
      // --- conv + SiLU
      const float aq = silu(wq0 * qs0 + wq1 * qs1 + wq2 * qs2 + wq3 * xq);
      qs0 = qs1; qs1 = qs2; qs2 = xq;
      if (tid < 128) {
        q_s[tid] = aq;
        v_s[tid] = silu(wv0 * vs0 + wv1 * vs1 + wv2 * vs2 + wv3 * xv);
        vs0 = vs1; vs1 = vs2; vs2 = xv;
      } else {
        k_s[tid - 128] = aq;
      }
      const float sq = warp_sum(aq * aq);
      if ((tid & 31) == 0) nrm[tid >> 5] = sq;
      if (tid == 0) {
        const float g = A * softplusf(aa + dtb);
        scal[0] = 1.f / (1.f + expf(-bb));   // beta
        scal[1] = g;
        scal[2] = expf(g);                    // decay
      }
      __syncthreads();                                                     // (1) q, k, v, norms
      // --- raw k^T S and q^T S for this thread's tile; raw q.k
      float ks[4] = {0.f, 0.f, 0.f, 0.f}, qsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float kk = k_s[kr * 16 + i], qq = q_s[kr * 16 + i];
        ks[0] += kk * st[i].x; ks[1] += kk * st[i].y; ks[2] += kk * st[i].z; ks[3] += kk * st[i].w;
        qsum[0] += qq * st[i].x; qsum[1] += qq * st[i].y; qsum[2] += qq * st[i].z; qsum[3] += qq * st[i].w;
      }
      *reinterpret_cast<float4*>(&red_k[kr][vc]) = make_float4(ks[0], ks[1], ks[2], ks[3]);
      *reinterpret_cast<float4*>(&red_q[kr][vc]) = make_float4(qsum[0], qsum[1], qsum[2], qsum[3]);
      float qk_part = tid < 128 ? q_s[tid] * k_s[tid] : 0.f;
      qk_part = warp_sum(qk_part);
      if ((tid & 31) == 0 && tid < 128) scal[4 + (tid >> 5)] = qk_part;
      const float iq = rsqrtf(nrm[0] + nrm[1] + nrm[2] + nrm[3] + 1e-6f) * inv_sqrt_d;
      const float ik = rsqrtf(nrm[4] + nrm[5] + nrm[6] + nrm[7] + 1e-6f);
      const float beta = scal[0], g = scal[1], decay = scal[2];
      __syncthreads();                                                     // (2) partial sums
      float o = 0.f;
      if (tid < 128) {
        float kS = 0.f, qS = 0.f;
#pragma unroll
        for (int g8 = 0; g8 < 8; ++g8) { kS += red_k[g8][tid]; qS += red_q[g8][tid]; }
        kS *= ik;
        qS *= iq;
        const float qk = (scal[4] + scal[5] + scal[6] + scal[7]) * (iq * ik);
        const float delta = (v_s[tid] - decay * kS) * beta;
        d_s[tid] = delta * ik;  // the state update multiplies by the raw key
        o = decay * qS + qk * delta;
        if (a.rec_k) {
          a.rec_k[(size_t(t) * a.Hv + h) * D + tid] = k_s[tid] * ik;
          a.rec_delta[(size_t(t) * a.Hv + h) * D + tid] = delta;
          if (tid == 0) a.rec_g[size_t(t) * a.Hv + h] = g;
        }
      }
      __syncthreads();                                                     // (3) delta
      // --- state update
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float kk = k_s[kr * 16 + i];
        st[i].x = decay * st[i].x + kk * d_s[vc + 0];
        st[i].y = decay * st[i].y + kk * d_s[vc + 1];
        st[i].z = decay * st[i].z + kk * d_s[vc + 2];
        st[i].w = decay * st[i].w + kk * d_s[vc + 3];
      }
      const int hrow = a.hist_row ? a.hist_row[t] : -1;
      if (hrow >= 0) {
        if (a.hist_rec) {  // conv-only history (MTP verify) skips the 64 KB state snapshot
          float* HS = a.hist_rec + ((size_t(hrow) * a.Hv + h) * D) * D;
#pragma unroll
          for (int i = 0; i < 16; ++i) *reinterpret_cast<float4*>(HS + (kr * 16 + i) * D + vc) = st[i];
        }
        __nv_bfloat16* hc = a.hist_conv + size_t(hrow) * a.C * (KW - 1);
        if (j == 0) {
          __nv_bfloat16* p = hc + size_t(qk_ch) * (KW - 1);
          p[0] = __float2bfloat16(qs0); p[1] = __float2bfloat16(qs1); p[2] = __float2bfloat16(qs2);
        }
        if (tid < 128) {
          __nv_bfloat16* p = hc + size_t(v_ch) * (KW - 1);
          p[0] = __float2bfloat16(vs0); p[1] = __float2bfloat16(vs1); p[2] = __float2bfloat16(vs2);
        }
      }
      // --- gated RMSNorm epilogue.  Its barrier also ends the token: every thread has finished
      // reading q/k/v/d of this token before the next one overwrites them, and ``ep`` is written
      // again only after barrier (1) of the next token.
      const float ob = __bfloat162float(__float2bfloat16(o));
      const float osq = warp_sum(tid < 128 ? ob * ob : 0.f);
      if ((tid & 31) == 0 && tid < 128) ep[tid >> 5] = osq;
      __syncthreads();                                                     // (4) output norm
      if (tid < 128) {
        const float ss = ep[0] + ep[1] + ep[2] + ep[3];
        const float y = ob * rsqrtf(ss / float(D) + a.eps) * __bfloat162float(a.norm_w[tid]) * silu(z);
        a.out[size_t(t) * (a.Hv * D) + h * D + tid] = __float2bfloat16(y);
      }
    }
    if (a.write_final) {
#pragma unroll
      for (int i = 0; i < 16; ++i) *reinterpret_cast<float4*>(S + (kr * 16 + i) * D + vc) = st[i];
      if (tid < 128) {
        __nv_bfloat16* cv = a.conv + (size_t(slot) * a.C + v_ch) * (KW - 1);
        cv[0] = __float2bfloat16(vs0); cv[1] = __float2bfloat16(vs1); cv[2] = __float2bfloat16(vs2);
      }
      if (j == r - 1) {
        // every value head re-read the untouched q/k window; commit it once, last
        cq[0] = __float2bfloat16(qs0); cq[1] = __float2bfloat16(qs1); cq[2] = __float2bfloat16(qs2);
      }
    }
    __syncthreads();
  }
  }  // items
}

__global__ void __launch_bounds__(kThreads) replay_commit_kernel(float* rec, int pool_slots, const int* slots,
                                                                 const float* keys, const float* deltas,
                                                                 const float* gs, const int* lens, int steps, int B,
                                                                 int Hv, int layer_rows) {
  const int h = blockIdx.x, b = blockIdx.y, l = blockIdx.z;
  const int tid = threadIdx.x, kr = tid >> 5, vc = (tid & 31) * 4;
  const int n = min(max(lens[b], 0), steps);
  if (n == 0) return;
  const int slot = slots[b];
  if (slot < 0 || slot >= pool_slots) {  // never write outside the pool: flag the batch as invalid
    if (tid == 0) atomicOr(&g_gdn_err, 4u);
    return;
  }
  float* S = rec + (((size_t(l) * pool_slots + slot) * Hv + h) * D) * D;
  float4 st[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) st[i] = *reinterpret_cast<const float4*>(S + (kr * 16 + i) * D + vc);
  for (int t = 0; t < n; ++t) {
    const size_t row = (size_t(l) * layer_rows + size_t(b) * steps + t) * Hv + h;
    const float e = expf(gs[row]);
    const float4 dl = *reinterpret_cast<const float4*>(deltas + row * D + vc);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float kk = keys[row * D + kr * 16 + i];
      st[i].x = e * st[i].x + kk * dl.x;
      st[i].y = e * st[i].y + kk * dl.y;
      st[i].z = e * st[i].z + kk * dl.z;
      st[i].w = e * st[i].w + kk * dl.w;
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) *reinterpret_cast<float4*>(S + (kr * 16 + i) * D + vc) = st[i];
}

__global__ void conv_commit_kernel(__nv_bfloat16* conv, int pool_slots, const __nv_bfloat16* hist, int hist_rows,
                                   const int* slots, const int* bounds, int steps, int elems) {
  const int b = blockIdx.x, l = blockIdx.y;
  const int slot = slots[b], bound = bounds[b];
  if (slot < 0 || slot >= pool_slots || bound < 0 || bound >= steps) {  // out of range: flag, write nothing
    if (threadIdx.x == 0) atomicOr(&g_gdn_err, 8u);
    return;
  }
  const int row = b * steps + bound;
  const __nv_bfloat16* src = hist + (size_t(l) * hist_rows + row) * elems;
  __nv_bfloat16* dst = conv + (size_t(l) * pool_slots + slot) * elems;
  for (int i = threadIdx.x; i < elems; i += blockDim.x) dst[i] = src[i];
}

void check_gdn(const at::Tensor& proj, const at::Tensor& rec, const at::Tensor& conv, int64_t dk, int64_t dv,
               int64_t hk, int64_t hv) {
  TORCH_CHECK(dk == D && dv == D, "CUDA GDN kernels handle key/value head dim 128");
  TORCH_CHECK(hv % hk == 0, "Hv must be a multiple of Hk");
  TORCH_CHECK((proj.scalar_type() == at::kBFloat16 || proj.scalar_type() == at::kFloat) && proj.is_contiguous(),
              "proj must be contiguous bf16 (or an fp32 accumulator)");
  TORCH_CHECK(rec.scalar_type() == at::kFloat && rec.is_contiguous() && rec.size(1) == hv, "bad recurrent pool");
  TORCH_CHECK(conv.scalar_type() == at::kBFloat16 && conv.is_contiguous() && conv.size(2) == KW - 1,
              "bad conv pool");
}

ScanArgs make_args(const at::Tensor& proj, const at::Tensor& slots, const at::Tensor& conv_w, const at::Tensor& A_log,
                   const at::Tensor& dt_bias, const at::Tensor& norm_w, at::Tensor& rec, at::Tensor& conv,
                   at::Tensor& out, int64_t hk, int64_t hv, double eps) {
  ScanArgs a = {};
  a.proj = proj.data_ptr();
  a.proj_stride = proj.size(1);
  a.slots = slots.data_ptr<int>();
  a.conv_w = reinterpret_cast<const __nv_bfloat16*>(conv_w.data_ptr());
  a.A_log = A_log.data_ptr<float>();
  a.dt_bias = dt_bias.data_ptr<float>();
  a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr());
  a.rec = rec.data_ptr<float>();
  a.conv = reinterpret_cast<__nv_bfloat16*>(conv.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.Hk = hk;
  a.Hv = hv;
  a.C = conv.size(1);
  a.eps = float(eps);
  a.write_final = true;
  TORCH_CHECK(a.C == 2 * hk * D + hv * D, "conv pool channel count mismatch");
  TORCH_CHECK(proj.size(1) >= a.C + hv * D + 2 * hv, "projection width mismatch");
  TORCH_CHECK(conv_w.scalar_type() == at::kBFloat16 && conv_w.size(0) == a.C && conv_w.size(1) == KW, "conv weight");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat, "A_log/dt_bias must be fp32");
  TORCH_CHECK(slots.scalar_type() == at::kInt, "slots must be int32");
  return a;
}

bool gdn_persist_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("ISB_GDN_PERSIST");
    return !(e && e[0] == '0');
  }();
  return on;
}

int gdn_num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <typename TIn>
void launch_scan_t(const ScanArgs& a, int64_t hk, int B, cudaStream_t st) {
  const int items = int(hk) * B;
  const int grid = 2 * gdn_num_sms();
  if (a.cu_seqlens == nullptr && a.hist_row == nullptr && gdn_persist_enabled() && items >= 2 * grid) {
    auto kern = gdn_scan_kernel<TIn, true>;
    static bool attr = false;
    if (!attr) {
      TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, D * D * 4) == cudaSuccess,
                  "persistent GDN smem attribute");
      attr = true;
    }
    launch_pdl(kern, dim3(grid), dim3(kThreads), D * D * 4, st, a, items);
    return;
  }
  launch_pdl(gdn_scan_kernel<TIn, false>, dim3(hk, B), dim3(kThreads), 0, st, a, 0);
}

void launch_scan(const ScanArgs& a, const at::Tensor& proj, int64_t hk, int B) {
  auto st = at::cuda::getCurrentCUDAStream();
  if (proj.scalar_type() == at::kFloat) launch_scan_t<float>(a, hk, B, st);
  else launch_scan_t<__nv_bfloat16>(a, hk, B, st);
}

}  // namespace

at::Tensor gdn_decode(const at::Tensor& proj, const at::Tensor& slots, const at::Tensor& conv_w, const at::Tensor& A_log,
                      const at::Tensor& dt_bias, const at::Tensor& norm_w, at::Tensor rec, at::Tensor conv, int64_t hk,
                      int64_t hv, int64_t dk, int64_t dv, double eps) {
  check_gdn(proj, rec, conv, dk, dv, hk, hv);
  const int B = proj.size(0);
  at::Tensor out = at::empty({B, hv * D}, proj.options().dtype(at::kBFloat16));
  if (B == 0) return out;
  ScanArgs a = make_args(proj, slots, conv_w, A_log, dt_bias, norm_w, rec, conv, out, hk, hv, eps);
  launch_scan(a, proj, hk, B);
  return out;
}

at::Tensor gdn_prefill(const at::Tensor& proj, const at::Tensor& cu_seqlens, const at::Tensor& slots,
                       const at::Tensor& conv_w, const at::Tensor& A_log, const at::Tensor& dt_bias,
                       const at::Tensor& norm_w, at::Tensor rec, at::Tensor conv, int64_t hk, int64_t hv, int64_t dk,
                       int64_t dv, double eps, int64_t max_seqlen) {
  check_gdn(proj, rec, conv, dk, dv, hk, hv);
  const int T = proj.size(0), B = slots.numel();
  at::Tensor out = at::empty({T, hv * D}, proj.options().dtype(at::kBFloat16));
  if (T == 0 || B == 0) return out;
  ScanArgs a = make_args(proj, slots, conv_w, A_log, dt_bias, norm_w, rec, conv, out, hk, hv, eps);
  a.cu_seqlens = cu_seqlens.data_ptr<int>();
  launch_scan(a, proj, hk, B);
  return out;
}

// Scan with per-token state history and/or replay records; optionally leaves the pool untouched.
at::Tensor gdn_scan_history(const at::Tensor& proj, const at::Tensor& cu_seqlens, const at::Tensor& slots,
                            const at::Tensor& conv_w, const at::Tensor& A_log, const at::Tensor& dt_bias,
                            const at::Tensor& norm_w, at::Tensor rec, at::Tensor conv, int64_t hk, int64_t hv,
                            double eps, bool write_final, const c10::optional<at::Tensor>& hist_row,
                            c10::optional<at::Tensor> hist_rec, c10::optional<at::Tensor> hist_conv,
                            c10::optional<at::Tensor> rec_k, c10::optional<at::Tensor> rec_delta,
                            c10::optional<at::Tensor> rec_g) {
  check_gdn(proj, rec, conv, D, D, hk, hv);
  const int T = proj.size(0), B = slots.numel();
  at::Tensor out = at::empty({T, hv * D}, proj.options().dtype(at::kBFloat16));
  if (T == 0 || B == 0) return out;
  ScanArgs a = make_args(proj, slots, conv_w, A_log, dt_bias, norm_w, rec, conv, out, hk, hv, eps);
  a.cu_seqlens = cu_seqlens.data_ptr<int>();
  a.write_final = write_final;
  if (hist_row.has_value()) {
    TORCH_CHECK(hist_conv.has_value(), "history needs a conv buffer (the recurrent one is optional)");
    a.hist_row = hist_row->data_ptr<int>();
    a.hist_rec = hist_rec.has_value() ? hist_rec->data_ptr<float>() : nullptr;
    a.hist_conv = reinterpret_cast<__nv_bfloat16*>(hist_conv->data_ptr());
  }
  if (rec_k.has_value()) {
    a.rec_k = rec_k->data_ptr<float>();
    a.rec_delta = rec_delta->data_ptr<float>();
    a.rec_g = rec_g->data_ptr<float>();
  }
  launch_scan(a, proj, hk, B);
  return out;
}

void gdn_replay_commit(at::Tensor rec, const at::Tensor& slots, const at::Tensor& keys, const at::Tensor& deltas,
                       const at::Tensor& gs, const at::Tensor& lens, int64_t steps) {
  TORCH_CHECK(rec.dim() == 5 && rec.size(3) == D && rec.size(4) == D, "recurrent pool must be [L, S, Hv, 128, 128]");
  const int L = rec.size(0), B = slots.numel(), Hv = rec.size(2);
  if (B == 0) return;
  // records are [L, rows, Hv, D] (rows >= B * steps; row b * steps + t of each layer is read)
  TORCH_CHECK(keys.dim() == 4 && keys.size(0) == L && keys.size(1) >= int64_t(B) * steps && keys.size(2) == Hv,
              "replay keys must be [L, rows >= B*steps, Hv, 128]");
  TORCH_CHECK(deltas.sizes() == keys.sizes() && gs.dim() == 3 && gs.size(1) == keys.size(1), "replay record shapes");
  at::Tensor k = keys.to(at::kFloat).contiguous(), d = deltas.to(at::kFloat).contiguous(),
             g = gs.to(at::kFloat).contiguous();
  at::Tensor sl = slots.to(at::kInt).contiguous(), ln = lens.to(at::kInt).contiguous();
  replay_commit_kernel<<<dim3(Hv, B, L), kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      rec.data_ptr<float>(), rec.size(1), sl.data_ptr<int>(), k.data_ptr<float>(), d.data_ptr<float>(),
      g.data_ptr<float>(), ln.data_ptr<int>(), int(steps), B, Hv, int(k.size(1)));
}

void gdn_conv_commit(at::Tensor conv, const at::Tensor& hist, const at::Tensor& slots, const at::Tensor& bounds,
                     int64_t steps) {
  TORCH_CHECK(conv.dim() == 4 && hist.dim() == 4, "conv pool [L,S,C,3], history [L,rows,C,3]");
  const int L = conv.size(0), B = slots.numel();
  if (B == 0) return;
  TORCH_CHECK(hist.size(0) == L && hist.size(1) >= int64_t(B) * steps && hist.size(2) == conv.size(2),
              "conv history must be [L, rows >= B*steps, C, 3]");
  at::Tensor sl = slots.to(at::kInt).contiguous(), bd = bounds.to(at::kInt).contiguous();
  at::Tensor h = hist.contiguous();
  conv_commit_kernel<<<dim3(B, L), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(conv.data_ptr()), conv.size(1),
      reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), h.size(1), sl.data_ptr<int>(), bd.data_ptr<int>(),
      int(steps), int(conv.size(2) * conv.size(3)));
}

int64_t gdn_error_word() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_gdn_err, sizeof(v));
  const unsigned int z = 0;
  cudaMemcpyToSymbol(g_gdn_err, &z, sizeof(z));
  return v;
}

// Device address of the error word (read by the per-step status kernel).
int64_t gdn_error_word_address() {
  void* p = nullptr;
  TORCH_CHECK(cudaGetSymbolAddress(&p, g_gdn_err) == cudaSuccess, "error word address");
  return reinterpret_cast<int64_t>(p);
}

}  // namespace isb
