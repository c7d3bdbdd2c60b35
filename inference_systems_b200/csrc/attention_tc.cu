// Tensor-core causal prefill attention over the paged KV cache (head_dim 256, GQA).
//
// One CTA per (tile of 128/G new tokens x the G query heads of one KV head, KV
// head, sequence): the G heads of a GQA group share every K/V block, so the MMA
// M dimension is tokens x heads = 128 rows.  Per block of 64 keys:
//   S  = Q K^T           tcgen05.mma M=128, N=64,  K=256  -> TMEM (double-buffered)
//   softmax (online)     warps 4-7, one TMEM lane (= query row) per thread
//   O += P V             tcgen05.mma M=128, N=256, K=64   -> TMEM
// Q and K arrive by TMA (128-byte swizzle, K-major).  V is the B operand of the
// second MMA with the key dimension as K, so it must be key-contiguous: warps
// 2-3 load each V block and write its transpose into shared memory in the same
// swizzled K-major layout (8x8 register transposes, 16-byte stores).  P is
// written by the softmax threads in that layout too.  Every wait is bounded
// (globaltimer): on expiry the kernel records an error, stops and frees TMEM.
// Parity (behaviour): flash-attn varlen prefill with a block table and the
// sigmoid output gate (``nanovllm/layers/attention.py:59-75``,
// ``nanovllm/models/qwen3_5.py:86,95``).

#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "common.cuh"
#include "launch.cuh"

namespace isb {
namespace {

constexpr int HD = 256;     // head dim
constexpr int KB = 64;      // keys per block
constexpr int MR = 128;     // MMA rows (tokens x heads)
constexpr int PAGE = 256;   // KV page
constexpr int Q_BYTES = MR * HD * 2;    // 4 swizzle-atom columns of 16 KB
constexpr int K_BYTES = KB * HD * 2;    // 4 atom columns of 8 KB
constexpr int VT_BYTES = HD * KB * 2;   // 256 rows x 128 B
constexpr int P_BYTES = MR * KB * 2;    // 128 rows x 128 B
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = Q_BYTES + 2 * K_BYTES + 2 * VT_BYTES + P_BYTES + BAR_BYTES + 1024;
constexpr uint32_t TMEM_COLS = 512;     // S0 [0,64) S1 [64,128) O [256,512)

__device__ unsigned int g_attn_tc_err;

struct TcArgs {
  const __nv_bfloat16* v_cache;  // [blocks, Hkv, 256, HD]
  const int* cu_q;
  const int* ctx_lens;
  const int* block_tables;
  int max_blocks;
  int Hq, Hkv;
  float scale_log2;  // softmax scale * log2(e)
  const __nv_bfloat16* gate;  // [T, Hq * HD] or null
  __nv_bfloat16* out;         // [T, Hq * HD]
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int G>
__global__ void __launch_bounds__(256, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK, TcArgs a) {
  constexpr int QT = MR / G;          // tokens per tile; G * QT <= 128 rows are used
  constexpr int QROWS = G * QT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;
  uint8_t* k_s = q_s + Q_BYTES;
  uint8_t* vt_s = k_s + 2 * K_BYTES;
  uint8_t* p_s = vt_s + 2 * VT_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + P_BYTES);
  uint64_t* qfull = bars;
  uint64_t* kfull = bars + 1;    // [2]
  uint64_t* vfull = bars + 3;    // [2]
  uint64_t* kvfree = bars + 5;   // [2]
  uint64_t* sfull = bars + 7;    // [2]
  uint64_t* sfree = bars + 9;    // [2]
  uint64_t* pready = bars + 11;
  uint64_t* pvdone = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  pdl_trigger();
  pdl_wait();  // q, gate and the new K/V rows come from the kernel right before
  const int qt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_start = a.cu_q[b], nq = a.cu_q[b + 1] - q_start;
  const int q0 = qt * QT;
  if (q0 >= nq) return;  // whole CTA, before any TMEM is taken
  const int past = a.ctx_lens[b] - nq;            // cached tokens before the first new one
  const int q_last = min(q0 + QT, nq) - 1;
  const int nkb = (past + q_last) / KB + 1;       // key blocks covering keys [0, past + q_last]
  const int* bt = a.block_tables + size_t(b) * a.max_blocks;

  if (threadIdx.x == 0) {
    mbar_init(qfull, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kfull[s], 1);
      mbar_init(&vfull[s], 64);
      mbar_init(&kvfree[s], 1);
      mbar_init(&sfull[s], 1);
      mbar_init(&sfree[s], 128);
    }
    mbar_init(pready, 128);
    mbar_init(pvdone, 1);
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    // ---------------------------------------------------- TMA: Q once, K blocks
    if (lane == 0) {
      mbar_arrive_expect_tx(qfull, QROWS * HD * 2);  // rows past QROWS stay unused
      for (int c = 0; c < 4; ++c) tma_load_3d(q_s + c * (Q_BYTES / 4), &tmQ, qfull, c * 64, kvh * G, q_start + q0);
      for (int j = 0; j < nkb; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kvfree[s], ((j >> 1) - 1) & 1)) { atomicOr(&g_attn_tc_err, 1u); break; }
        const int key0 = j * KB;
        const int row = (bt[key0 / PAGE] * a.Hkv + kvh) * PAGE + key0 % PAGE;
        mbar_arrive_expect_tx(&kfull[s], K_BYTES);
        for (int c = 0; c < 4; ++c) tma_load_2d(k_s + s * K_BYTES + c * (K_BYTES / 4), &tmK, &kfull[s], c * 64, row);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(MR, KB), idO = idesc_bf16_f32(MR, HD);
      bool ok = mbar_wait(qfull, 0);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&kfull[s], (j >> 1) & 1)) return false;
        if (j >= 2 && !mbar_wait(&sfree[s], ((j >> 1) - 1) & 1)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t ad = smem_desc_sw128(q_s + (k >> 2) * (Q_BYTES / 4)) + 2 * (k & 3);
          const uint64_t bd = smem_desc_sw128(k_s + s * K_BYTES + (k >> 2) * (K_BYTES / 4)) + 2 * (k & 3);
          mma_bf16(tmem + s * KB, ad, bd, idS, k > 0 ? 1u : 0u);
        }
        mma_commit(&sfull[s]);
        return true;
      };
      ok = ok && issue_s(0);
      for (int j = 0; ok && j < nkb; ++j) {
        if (j + 1 < nkb && !issue_s(j + 1)) { ok = false; break; }
        const int s = j & 1;
        if (!mbar_wait(pready, j & 1) || !mbar_wait(&vfull[s], (j >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < KB / 16; ++k) {
          const uint64_t ad = smem_desc_sw128(p_s) + 2 * k;
          const uint64_t bd = smem_desc_sw128(vt_s + s * VT_BYTES) + 2 * k;
          mma_bf16(tO, ad, bd, idO, (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&kvfree[s]);
        mma_commit(pvdone);
      }
      if (!ok) atomicOr(&g_attn_tc_err, 2u);
    }
  } else if (warp < 4) {
    // ---------------------------------------------------- V^T producers (64 threads)
    const int vt = threadIdx.x - 64;
    for (int j = 0; j < nkb; ++j) {
      const int s = j & 1;
      if (j >= 2 && !mbar_wait(&kvfree[s], ((j >> 1) - 1) & 1)) { atomicOr(&g_attn_tc_err, 4u); break; }
      const int key0 = j * KB;
      const __nv_bfloat16* vsrc =
          a.v_cache + ((size_t(bt[key0 / PAGE]) * a.Hkv + kvh) * PAGE + key0 % PAGE) * HD;
      uint8_t* dst = vt_s + s * VT_BYTES;
      // 8 keys x 8 dims micro-tiles; V^T row d holds 64 keys (128 B, swizzled 16-byte chunks)
      for (int m = vt; m < (KB / 8) * (HD / 8); m += 64) {
        const int kc = m & 7, dc = m >> 3;
        uint4 in[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) in[i] = *reinterpret_cast<const uint4*>(vsrc + size_t(kc * 8 + i) * HD + dc * 8);
        // element (key i, dim x) of the micro-tile; x is a compile-time constant after unrolling
        auto e = [&](int i, int x) -> uint32_t {
          const uint32_t w = x < 2 ? in[i].x : x < 4 ? in[i].y : x < 6 ? in[i].z : in[i].w;
          return (x & 1) ? (w >> 16) : (w & 0xFFFFu);
        };
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          const int d = dc * 8 + x;
          uint4 o;
          o.x = e(0, x) | (e(1, x) << 16);
          o.y = e(2, x) | (e(3, x) << 16);
          o.z = e(4, x) | (e(5, x) << 16);
          o.w = e(6, x) | (e(7, x) << 16);
          *reinterpret_cast<uint4*>(dst + d * 128 + ((kc ^ (d & 7)) * 16)) = o;
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&vfull[s]);
    }
  } else {
    // ---------------------------------------------------- softmax + epilogue (warps 4..7)
    const int r = threadIdx.x - 128;                       // query row == TMEM lane
    const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;
    const int q_local = q0 + r / G;
    const bool row_ok = r < QROWS && q_local < nq;
    const int qpos = past + q_local;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&sfull[s], (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      float sc[KB];
      tmem_ld32(tmem + s * KB + lane_base, sc);
      tmem_ld32(tmem + s * KB + 32 + lane_base, sc + 32);
      tc_fence_before();
      mbar_arrive(&sfree[s]);
      const int key0 = j * KB;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < KB; ++c) {
        float x = sc[c] * a.scale_log2;
        if (!row_ok) x = 0.f;
        else if (key0 + c > qpos) x = -INFINITY;
        sc[c] = x;
        mx = fmaxf(mx, x);
      }
      const float m_new = fmaxf(m, mx);  // finite: key 0 is visible to every row
      const float alpha = exp2f(m - m_new);
      float sum = 0.f;
      uint32_t pk[KB / 2];
#pragma unroll
      for (int c = 0; c < KB; c += 2) {
        const float p0 = exp2f(sc[c] - m_new), p1 = exp2f(sc[c + 1] - m_new);
        sum += p0 + p1;
        pk[c / 2] = pack_bf16(p0, p1);
      }
      l = l * alpha + sum;
      m = m_new;
      if (j > 0) {
        // P(j-1) and O must be free: the previous P V has completed
        if (!mbar_wait(pvdone, (j - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha < 1.f)) {
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            float o[32];
            tmem_ld32(tO + c + lane_base, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + c + lane_base, o);
          }
        }
      }
      uint8_t* prow = p_s + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) * 16)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(pready);
    }
    if (ok && !mbar_wait(pvdone, (nkb - 1) & 1)) ok = false;
    if (!ok) atomicOr(&g_attn_tc_err, 8u);
    tc_fence_after();
    const float inv_l = (ok && l > 0.f) ? 1.f / l : 0.f;
    const int t = q_start + q_local, h = kvh * G + r % G;
    __nv_bfloat16* orow = a.out + (size_t(t) * a.Hq + h) * HD;
    const __nv_bfloat16* grow = a.gate ? a.gate + (size_t(t) * a.Hq + h) * HD : nullptr;
#pragma unroll 1
    for (int c = 0; c < HD; c += 32) {
      float o[32];
      tmem_ld32(tO + c + lane_base, o);  // warp-collective: every lane, valid row or not
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 pkd;
          uint32_t* w = reinterpret_cast<uint32_t*>(&pkd);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float v0 = o[i + 2 * e] * inv_l, v1 = o[i + 2 * e + 1] * inv_l;
            if (grow) {
              v0 *= sigmoidf_(__bfloat162float(grow[c + i + 2 * e]));
              v1 *= sigmoidf_(__bfloat162float(grow[c + i + 2 * e + 1]));
            }
            w[e] = pack_bf16(v0, v1);
          }
          *reinterpret_cast<uint4*>(orow + c + i) = pkd;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_tc() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
                    q == cudaDriverEntryPointSuccess && p,
                "cannot resolve cuTensorMapEncodeTiled");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

template <int G>
void launch_tc(const at::Tensor& q, const at::Tensor& kc, const TcArgs& a, int B, int max_seqlen_q, cudaStream_t st) {
  constexpr int QT = MR / G;
  const int T = q.size(0);
  CUtensorMap tq, tk;
  {
    cuuint64_t dims[3] = {cuuint64_t(HD), cuuint64_t(a.Hq), cuuint64_t(T)};
    cuuint64_t strides[2] = {cuuint64_t(HD) * 2, cuuint64_t(a.Hq) * HD * 2};
    cuuint32_t box[3] = {64, cuuint32_t(G), cuuint32_t(QT)};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = encode_fn_tc()(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q.data_ptr(), dims, strides, box, es,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (q) failed: ", int(r));
  }
  {
    const int64_t rows = kc.size(0) * kc.size(1) * kc.size(2);
    cuuint64_t dims[2] = {cuuint64_t(HD), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(HD) * 2};
    cuuint32_t box[2] = {64, KB};
    cuuint32_t es[2] = {1, 1};
    CUresult r = encode_fn_tc()(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kc.data_ptr(), dims, strides, box, es,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (k) failed: ", int(r));
  }
  auto kern = attn_prefill_tc_kernel<G>;
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) == cudaSuccess,
                "tc attention smem attribute");
    attr = true;
  }
  const dim3 grid((max_seqlen_q + QT - 1) / QT, a.Hkv, B);
  launch_pdl(kern, grid, dim3(256), SMEM_BYTES, st, tq, tk, a);
}

}  // namespace

bool attention_prefill_tc_supported(int64_t hd, int64_t hq, int64_t hkv) {
  if (hd != HD || hq % hkv) return false;
  const int64_t g = hq / hkv;
  return g == 1 || g == 2 || g == 3 || g == 4 || g == 6 || g == 8;
}

at::Tensor attention_prefill_tc(const at::Tensor& q, const at::Tensor& gate, const at::Tensor& kc, const at::Tensor& vc,
                                const at::Tensor& cu_q, const at::Tensor& ctx_lens, const at::Tensor& block_tables,
                                double scale, bool gated, int64_t max_seqlen_q) {
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous() && q.scalar_type() == at::kBFloat16, "q must be [T, Hq, 256] bf16");
  TORCH_CHECK(kc.dim() == 4 && kc.size(2) == PAGE && kc.size(3) == HD && kc.is_contiguous() && vc.is_contiguous(),
              "KV cache must be [blocks, Hkv, 256, 256]");
  const int T = q.size(0), Hq = q.size(1), Hkv = kc.size(1), B = ctx_lens.numel();
  TORCH_CHECK(attention_prefill_tc_supported(q.size(2), Hq, Hkv), "unsupported head layout for tensor-core prefill");
  at::Tensor out = at::empty({T, Hq * HD}, q.options());
  if (T == 0 || B == 0) return out;
  TcArgs a = {};
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr());
  a.cu_q = cu_q.data_ptr<int>();
  a.ctx_lens = ctx_lens.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.max_blocks = block_tables.size(1);
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.scale_log2 = float(scale) * 1.4426950408889634f;
  a.gate = gated ? reinterpret_cast<const __nv_bfloat16*>(gate.data_ptr()) : nullptr;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  auto st = at::cuda::getCurrentCUDAStream();
  switch (Hq / Hkv) {
    case 1: launch_tc<1>(q, kc, a, B, int(max_seqlen_q), st); break;
    case 2: launch_tc<2>(q, kc, a, B, int(max_seqlen_q), st); break;
    case 3: launch_tc<3>(q, kc, a, B, int(max_seqlen_q), st); break;
    case 4: launch_tc<4>(q, kc, a, B, int(max_seqlen_q), st); break;
    case 6: launch_tc<6>(q, kc, a, B, int(max_seqlen_q), st); break;
    case 8: launch_tc<8>(q, kc, a, B, int(max_seqlen_q), st); break;
    default: TORCH_CHECK(false, "unsupported GQA group");
  }
  return out;
}

int64_t attn_tc_error_word() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_attn_tc_err, sizeof(v));
  const unsigned int z = 0;
  cudaMemcpyToSymbol(g_attn_tc_err, &z, sizeof(z));
  return v;
}

}  // namespace isb
