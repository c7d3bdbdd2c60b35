// Tensor-core causal prefill attention over the paged KV cache (head_dim 256, GQA).
//
// One CTA per (tile of 128/G new tokens x the G query heads of one KV head, KV
// head, sequence): the G heads of a GQA group share every K/V block, so the MMA
// M dimension is tokens x heads = 128 rows.  Per block of 64 keys:
//   S  = Q K^T           tcgen05.mma M=128, N=64,  K=256  -> TMEM (double-buffered)
//   softmax (online)     warps 4-7, one TMEM lane (= query row) per thread
//   O += P V             tcgen05.mma M=128, N=256, K=64   -> TMEM
// Q, K and V arrive by TMA (128-byte swizzle).  K is the K-major B operand of the first MMA;
// V is the B operand of the second in MN-major form, read straight from its tile (a swizzled
// [64 keys][64 dims] box is the canonical MN-major layout: dim blocks one box apart, key
// groups of 8 one 1024-byte atom apart), so no transpose is needed.  P is written by the
// softmax threads (K-major, swizzled) into one of two buffers, so the softmax of block j+1
// overlaps P V of block j.  The running maximum is raised only when a row's block maximum
// exceeds it by more than 8 (log2 units): P entries stay <= 2^8, and O is rescaled in tensor
// memory only on those raises.  Every wait is bounded (globaltimer): on expiry the kernel
// records an error, stops and frees TMEM.
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
constexpr int V_BYTES = KB * HD * 2;    // 4 boxes of [64 keys x 128 B]
constexpr int P_BYTES = MR * KB * 2;    // 128 rows x 128 B
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = Q_BYTES + 2 * K_BYTES + 2 * V_BYTES + 2 * P_BYTES + BAR_BYTES + 1024;
constexpr float kRescaleLog2 = 8.f;     // lazy-rescale threshold of the running maximum
constexpr uint32_t TMEM_COLS = 512;     // S0 [0,64) S1 [64,128) O [256,512)

__device__ unsigned int g_attn_tc_err;

struct TcArgs {
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

// MN-major operand, 128-byte swizzle: 64-element blocks along M/N are ``lbo`` bytes apart,
// groups of 8 rows along K are 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(const void* tile, uint32_t lbo) {
  const uint64_t addr = smem_u32(tile);
  uint64_t d = (addr >> 4) & 0x3FFFull;
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= (1024ull >> 4) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

template <int G>
__global__ void __launch_bounds__(256, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, TcArgs a) {
  constexpr int QT = MR / G;          // tokens per tile; G * QT <= 128 rows are used
  constexpr int QROWS = G * QT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;
  uint8_t* k_s = q_s + Q_BYTES;
  uint8_t* v_s = k_s + 2 * K_BYTES;
  uint8_t* p_s = v_s + 2 * V_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + 2 * P_BYTES);
  uint64_t* qfull = bars;
  uint64_t* kfull = bars + 1;    // [2]
  uint64_t* vfull = bars + 3;    // [2]
  uint64_t* kvfree = bars + 5;   // [2]
  uint64_t* sfull = bars + 7;    // [2]
  uint64_t* sfree = bars + 9;    // [2]
  uint64_t* pready = bars + 11;  // [2]
  uint64_t* pvdone = bars + 13;  // [2]
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
      mbar_init(&vfull[s], 1);
      mbar_init(&kvfree[s], 1);
      mbar_init(&sfull[s], 1);
      mbar_init(&sfree[s], 128);
      mbar_init(&pready[s], 128);
      mbar_init(&pvdone[s], 1);
    }
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    // ---------------------------------------------------- TMA: Q once, K and V blocks
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
        mbar_arrive_expect_tx(&vfull[s], V_BYTES);
        for (int c = 0; c < 4; ++c) tma_load_2d(v_s + s * V_BYTES + c * (V_BYTES / 4), &tmV, &vfull[s], c * 64, row);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(MR, KB);
      constexpr uint32_t idO = idesc_bf16_f32(MR, HD) | (1u << 16);  // B = V, MN-major
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
        if (!mbar_wait(&pready[s], (j >> 1) & 1) || !mbar_wait(&vfull[s], (j >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < KB / 16; ++k) {
          const uint64_t ad = smem_desc_sw128(p_s + s * P_BYTES) + 2 * k;
          const uint64_t bd = smem_desc_mn_sw128(v_s + s * V_BYTES + k * 2048, V_BYTES / 4);
          mma_bf16(tO, ad, bd, idO, (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&kvfree[s]);
        mma_commit(&pvdone[s]);
      }
      if (!ok) atomicOr(&g_attn_tc_err, 2u);
    }
  } else if (warp < 4) {
    // warps 2-3: idle (K and V both arrive by TMA)
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
      // the running maximum moves only when this block's exceeds it by more than 2^8 (the first
      // block always sets it: key 0 is visible to every row, so it is finite from then on)
      const bool raise = mx > m + kRescaleLog2;
      const float m_new = raise ? mx : m;
      const float alpha = raise ? exp2f(m - m_new) : 1.f;
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
      const int pb = j & 1;
      if (j > 0) {
        const bool rescale = __any_sync(0xffffffffu, alpha < 1.f);
        if (rescale) {
          // O is rescaled in place: every earlier P V (the last one, j-1, included) has completed
          if (!mbar_wait(&pvdone[(j - 1) & 1], ((j - 1) >> 1) & 1)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            float o[32];
            tmem_ld32(tO + c + lane_base, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tO + c + lane_base, o);
          }
        } else if (j > 1) {
          // P buffer pb is free once P V of block j-2 has completed
          if (!mbar_wait(&pvdone[pb], ((j - 2) >> 1) & 1)) { ok = false; break; }
          tc_fence_after();
        }
      }
      uint8_t* prow = p_s + pb * P_BYTES + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) * 16)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&pready[pb]);
    }
    if (ok && !mbar_wait(&pvdone[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1)) ok = false;
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

// ------------------------------------------------------------------ decode
// Persistent split-KV decode: one CTA per SM walks work items (key chunk of 128 tokens,
// sequence, KV head), chunk-major so the round-robin assignment spreads the non-empty
// items evenly.  Per item, with the G query heads of the KV head as the N = 16 (zero-padded)
// dimension:
//   S^T = K Q^T        tcgen05.mma M=128 keys, N=16, K=256        -> TMEM (double-buffered)
//   softmax            warps 2-5, one key per thread; per-head max / sum across the 4 warps
//   O^T = V^T P^T      2 x tcgen05.mma M=128 dims, N=16, K=128 keys -> TMEM (double-buffered)
// V is the A operand in MN-major form, read straight from its TMA tile (a 128-byte-swizzled
// [keys][64 dims] box is exactly the canonical MN-major layout: dim blocks of 64 one box
// (16 KB) apart, key groups of 8 one 1024-byte atom apart), so no transpose is needed.
// K and V tiles (64 KB each) stream through a 3-slot TMA ring that runs across items.
// The kernel writes unnormalised partials (o, max, sum) per (sequence, head, chunk); the
// split-KV combine kernel merges them and applies the output gate.  Key rows past the
// context inside the last tile are masked in the softmax, and their V rows are zeroed in
// shared memory before the P V product (stale cache rows may hold any bit pattern).
constexpr int DT = 128;                       // keys per tile (two tiles per page)
constexpr int KV_TILE = DT * HD * 2;          // 64 KB: 4 boxes of [128 rows x 128 B]
constexpr int NSLOT = 3;
constexpr int QD_BYTES = 16 * HD * 2;         // 4 blocks of [16 rows x 128 B]
constexpr int PD_BYTES = 16 * DT * 2;         // 2 blocks of [16 rows x 128 B]
constexpr int DEC_BAR_BYTES = 512;
constexpr int DEC_SMEM = NSLOT * KV_TILE + 2 * QD_BYTES + 2 * PD_BYTES + DEC_BAR_BYTES + 1024;
constexpr uint32_t DEC_TMEM_COLS = 128;       // S [0,32) (2 x 16), O [32,96) (2 x 2 x 16)

struct DecArgs {
  const int* ctx_lens;
  const int* block_tables;
  int max_blocks;
  int B, Hq, Hkv;
  float scale_log2;
  float* part_o;    // [B, Hq, max_chunks, HD]
  float* part_ml;   // [B, Hq, max_chunks, 2]
  int max_chunks;
  int nitems;       // max_chunks * B * Hkv
};

__device__ __forceinline__ void bar_sync_consumers() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int G>
__global__ void __launch_bounds__(192, 1)
    attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, DecArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kv_s = smem;
  uint8_t* q_s = kv_s + NSLOT * KV_TILE;
  uint8_t* p_s = q_s + 2 * QD_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + 2 * PD_BYTES);
  uint64_t* full = bars;        // [3] tile landed
  uint64_t* slotfree = bars + 3;  // [3] tile consumed by its MMA
  uint64_t* qfull = bars + 6;   // [2]
  uint64_t* qfree = bars + 8;   // [2]
  uint64_t* sfull = bars + 10;  // [2]
  uint64_t* sfree = bars + 12;  // [2]
  uint64_t* pfull = bars + 14;  // [2]
  uint64_t* pfree = bars + 16;  // [2]
  uint64_t* ofull = bars + 18;  // [2]
  uint64_t* ofree = bars + 20;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  float* red = reinterpret_cast<float*>(bars + 32);  // [2][4 warps][8 heads]

  pdl_trigger();
  pdl_wait();  // q and the new K/V rows come from the kernel right before
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Q and P rows >= G stay zero: TMA and the softmax write rows < G only
  for (int i = threadIdx.x; i < (2 * QD_BYTES + 2 * PD_BYTES) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(q_s)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&slotfree[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qfree[s], 1);
      mbar_init(&sfull[s], 1);
      mbar_init(&sfree[s], 128);
      mbar_init(&pfull[s], 128);
      mbar_init(&pfree[s], 1);
      mbar_init(&ofull[s], 1);
      mbar_init(&ofree[s], 128);
    }
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) tmem_alloc(tmem_slot, DEC_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int BH = a.B * a.Hkv;
  // item -> (sequence, KV head, chunk); false when the chunk starts past the context
  auto item = [&](int it, int& b, int& kvh, int& chunk, int& n) -> bool {
    chunk = it / BH;
    const int rem = it - chunk * BH;
    b = rem / a.Hkv;
    kvh = rem - b * a.Hkv;
    n = min(DT, a.ctx_lens[b] - chunk * DT);
    return n > 0;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int L = 0, j = 0;
      bool ok = true;
      for (int it = blockIdx.x; ok && it < a.nitems; it += gridDim.x) {
        int b, kvh, chunk, n;
        if (!item(it, b, kvh, chunk, n)) continue;
        const int qb = j & 1;
        if (j >= 2 && !mbar_wait(&qfree[qb], ((j >> 1) - 1) & 1)) { ok = false; break; }
        mbar_arrive_expect_tx(&qfull[qb], G * HD * 2);
        for (int c = 0; c < 4; ++c)
          tma_load_2d(q_s + qb * QD_BYTES + c * 2048, &tmQ, &qfull[qb], c * 64, b * a.Hq + kvh * G);
        const int key0 = chunk * DT;
        const int row = (a.block_tables[size_t(b) * a.max_blocks + key0 / PAGE] * a.Hkv + kvh) * PAGE + key0 % PAGE;
        for (int kv = 0; kv < 2; ++kv, ++L) {
          const int s = L % NSLOT, u = L / NSLOT;
          if (u >= 1 && !mbar_wait(&slotfree[s], (u - 1) & 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], KV_TILE);
          const CUtensorMap* tm = kv ? &tmV : &tmK;
          for (int c = 0; c < 4; ++c) tma_load_2d(kv_s + s * KV_TILE + c * (KV_TILE / 4), tm, &full[s], c * 64, row);
        }
        ++j;
      }
      if (!ok) atomicOr(&g_attn_tc_err, 0x10u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(128, 16);
      constexpr uint32_t idO = idesc_bf16_f32(128, 16) | (1u << 15);  // A = V^T, MN-major
      auto issue_s = [&](int j, int L) -> bool {
        const int b2 = j & 1, s = L % NSLOT;
        if (!mbar_wait(&qfull[b2], (j >> 1) & 1)) return false;
        if (!mbar_wait(&full[s], (L / NSLOT) & 1)) return false;
        if (j >= 2 && !mbar_wait(&sfree[b2], ((j >> 1) - 1) & 1)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t ad = smem_desc_sw128(kv_s + s * KV_TILE + (k >> 2) * (KV_TILE / 4)) + 2 * (k & 3);
          const uint64_t bd = smem_desc_sw128(q_s + b2 * QD_BYTES + (k >> 2) * 2048) + 2 * (k & 3);
          mma_bf16(tmem + b2 * 16, ad, bd, idS, k > 0 ? 1u : 0u);
        }
        mma_commit(&sfull[b2]);
        mma_commit(&slotfree[s]);
        mma_commit(&qfree[b2]);
        return true;
      };
      auto issue_pv = [&](int j, int L) -> bool {
        const int b2 = j & 1, s = L % NSLOT;
        if (!mbar_wait(&pfull[b2], (j >> 1) & 1)) return false;
        if (!mbar_wait(&full[s], (L / NSLOT) & 1)) return false;
        if (j >= 2 && !mbar_wait(&ofree[b2], ((j >> 1) - 1) & 1)) return false;
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int ks = 0; ks < DT / 16; ++ks) {
            const uint64_t ad = smem_desc_mn_sw128(kv_s + s * KV_TILE + 2 * h * (KV_TILE / 4) + ks * 2048, KV_TILE / 4);
            const uint64_t bd = smem_desc_sw128(p_s + b2 * PD_BYTES + (ks >> 2) * 2048) + 2 * (ks & 3);
            mma_bf16(tmem + 32 + b2 * 32 + h * 16, ad, bd, idO, ks > 0 ? 1u : 0u);
          }
        mma_commit(&ofull[b2]);
        mma_commit(&slotfree[s]);
        mma_commit(&pfree[b2]);
        return true;
      };
      // In order, S then P V per item: P V frees the V slot as early as possible, and the ring
      // (K of item j+1 waits for the slot of V of item j-1) keeps up to three tiles in flight.
      // Issuing S of the next item first would make P V wait for that item's K to land.
      int L = 0, j = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < a.nitems; it += gridDim.x) {
        int b, kvh, chunk, n;
        if (!item(it, b, kvh, chunk, n)) continue;
        if (!issue_s(j, L) || !issue_pv(j, L + 1)) { ok = false; break; }
        L += 2;
        ++j;
      }
      if (!ok) atomicOr(&g_attn_tc_err, 0x20u);
    }
  } else {
    // ------------------------------------------------------------ softmax + partials (warps 2..5)
    const int quad = warp & 3;             // TMEM lane quadrant of this warp
    const int r = quad * 32 + lane;        // key row of S^T, dim row of O^T
    const uint32_t lane_base = uint32_t(quad * 32) << 16;
    int L = 0, j = 0;
    bool ok = true;
    int pb_ = 0, pkvh = 0, pchunk = 0;
    float pm[G], pl[G];
    // A failed wait clears ``ok`` and later waits are skipped, but every thread keeps the same
    // sequence of named barriers and warp-collective TMEM loads, so nothing waits forever.
    auto wait = [&](uint64_t* bar, uint32_t parity) { ok = ok && mbar_wait(bar, parity); };
    auto emit = [&](int jj) {              // partials of the item before
      const int b2 = jj & 1;
      wait(&ofull[b2], (jj >> 1) & 1);
      __syncwarp();
      tc_fence_after();
      float o0[16], o1[16];
      tmem_ld16(tmem + 32 + b2 * 32 + lane_base, o0);
      tmem_ld16(tmem + 32 + b2 * 32 + 16 + lane_base, o1);
      tc_fence_before();
      mbar_arrive(&ofree[b2]);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const size_t base = (size_t(pb_) * a.Hq + pkvh * G + g) * a.max_chunks + pchunk;
        a.part_o[base * HD + r] = o0[g];
        a.part_o[base * HD + 128 + r] = o1[g];
        if (r == g) {
          a.part_ml[base * 2 + 0] = pm[g] * 0.6931471805599453f;  // back to natural-log units
          a.part_ml[base * 2 + 1] = pl[g];
        }
      }
    };
    for (int it = blockIdx.x; it < a.nitems; it += gridDim.x) {
      int b, kvh, chunk, n;
      if (!item(it, b, kvh, chunk, n)) continue;
      const int b2 = j & 1;
      wait(&sfull[b2], (j >> 1) & 1);
      __syncwarp();
      tc_fence_after();
      float sv[16];
      tmem_ld16(tmem + b2 * 16 + lane_base, sv);
      tc_fence_before();
      mbar_arrive(&sfree[b2]);
      const bool valid = r < n;
      float x[G], m[G], l[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        x[g] = valid ? sv[g] * a.scale_log2 : -INFINITY;
        const float mx = warp_max(x[g]);
        if (lane == 0) red[quad * 8 + g] = mx;
      }
      bar_sync_consumers();
#pragma unroll
      for (int g = 0; g < G; ++g) {
        m[g] = fmaxf(fmaxf(red[g], red[8 + g]), fmaxf(red[16 + g], red[24 + g]));  // finite: key 0 is valid
        x[g] = valid ? exp2f(x[g] - m[g]) : 0.f;
        const float sm = warp_sum(x[g]);
        if (lane == 0) red[32 + quad * 8 + g] = sm;
      }
      if (j >= 2) wait(&pfree[b2], ((j >> 1) - 1) & 1);
      uint8_t* prow = p_s + b2 * PD_BYTES + (r >> 6) * 2048;
      const int pc = (r & 63) >> 3;
#pragma unroll
      for (int g = 0; g < G; ++g)
        *reinterpret_cast<__nv_bfloat16*>(prow + g * 128 + ((pc ^ g) * 16) + (r & 7) * 2) = __float2bfloat16(x[g]);
      if (n < DT) {
        // last tile of the sequence: zero the V rows past the context before P V reads them
        const int vs = (L + 1) % NSLOT;
        wait(&full[vs], ((L + 1) / NSLOT) & 1);
        if (r >= n) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 8; ++i)
              *reinterpret_cast<uint4*>(kv_s + vs * KV_TILE + c * (KV_TILE / 4) + r * 128 + i * 16) =
                  make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&pfull[b2]);
      bar_sync_consumers();
#pragma unroll
      for (int g = 0; g < G; ++g) l[g] = (red[32 + g] + red[40 + g]) + (red[48 + g] + red[56 + g]);
      if (j > 0) emit(j - 1);
      pb_ = b; pkvh = kvh; pchunk = chunk;
#pragma unroll
      for (int g = 0; g < G; ++g) { pm[g] = m[g]; pl[g] = l[g]; }
      L += 2;
      ++j;
    }
    if (j > 0) emit(j - 1);
    if (!ok) atomicOr(&g_attn_tc_err, 0x40u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, DEC_TMEM_COLS);
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
void launch_tc(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const TcArgs& a, int B,
               int max_seqlen_q, cudaStream_t st) {
  constexpr int QT = MR / G;
  const int T = q.size(0);
  CUtensorMap tq, tk, tv;
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
    r = encode_fn_tc()(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, vc.data_ptr(), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (v) failed: ", int(r));
  }
  auto kern = attn_prefill_tc_kernel<G>;
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) == cudaSuccess,
                "tc attention smem attribute");
    attr = true;
  }
  const dim3 grid((max_seqlen_q + QT - 1) / QT, a.Hkv, B);
  launch_pdl(kern, grid, dim3(256), SMEM_BYTES, st, tq, tk, tv, a);
}

template <int G>
void launch_dec_tc(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const DecArgs& a,
                   cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  {
    cuuint64_t dims[2] = {cuuint64_t(HD), cuuint64_t(q.size(0)) * cuuint64_t(a.Hq)};
    cuuint64_t strides[1] = {cuuint64_t(HD) * 2};
    cuuint32_t box[2] = {64, cuuint32_t(G)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = encode_fn_tc()(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q.data_ptr(), dims, strides, box, es,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (decode q) failed: ", int(r));
  }
  const int64_t rows = kc.size(0) * kc.size(1) * kc.size(2);
  for (int w = 0; w < 2; ++w) {
    cuuint64_t dims[2] = {cuuint64_t(HD), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(HD) * 2};
    cuuint32_t box[2] = {64, DT};
    cuuint32_t es[2] = {1, 1};
    CUresult r = encode_fn_tc()(w ? &tv : &tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (w ? vc : kc).data_ptr(), dims,
                                strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (decode kv) failed: ", int(r));
  }
  auto kern = attn_decode_tc_kernel<G>;
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM) == cudaSuccess,
                "tc decode attention smem attribute");
    attr = true;
  }
  static int sms = 0;
  if (!sms) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int grid = std::max(1, std::min(sms, a.nitems));
  launch_pdl(kern, dim3(grid), dim3(192), DEC_SMEM, st, tq, tk, tv, a);
}

}  // namespace

bool attention_decode_tc_supported(int64_t hd, int64_t hq, int64_t hkv) {
  return hd == HD && hq % hkv == 0 && hq / hkv >= 1 && hq / hkv <= 8 && hq / hkv != 5 && hq / hkv != 7;
}

// Split-KV partials for 128-key chunks (chunk c of sequence b covers keys [128c, 128c+128));
// ``part_o`` [B, Hq, max_chunks, 256] and ``part_ml`` [B, Hq, max_chunks, 2] fp32, merged by
// the split-KV combine kernel.
void attention_decode_tc_partials(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc,
                                  const at::Tensor& ctx_lens, const at::Tensor& block_tables, double scale,
                                  at::Tensor& part_o, at::Tensor& part_ml, int max_chunks) {
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous() && q.scalar_type() == at::kBFloat16, "q must be [B, Hq, 256] bf16");
  TORCH_CHECK(kc.dim() == 4 && kc.size(2) == PAGE && kc.size(3) == HD && kc.is_contiguous() && vc.is_contiguous(),
              "KV cache must be [blocks, Hkv, 256, 256]");
  const int B = q.size(0), Hq = q.size(1), Hkv = kc.size(1);
  TORCH_CHECK(attention_decode_tc_supported(q.size(2), Hq, Hkv), "unsupported head layout for tensor-core decode");
  TORCH_CHECK(max_chunks == block_tables.size(1) * (PAGE / DT), "max_chunks must cover the block table");
  DecArgs a = {};
  a.ctx_lens = ctx_lens.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.max_blocks = block_tables.size(1);
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.scale_log2 = float(scale) * 1.4426950408889634f;
  a.part_o = part_o.data_ptr<float>();
  a.part_ml = part_ml.data_ptr<float>();
  a.max_chunks = max_chunks;
  a.nitems = max_chunks * B * Hkv;
  if (B == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  switch (Hq / Hkv) {
    case 1: launch_dec_tc<1>(q, kc, vc, a, st); break;
    case 2: launch_dec_tc<2>(q, kc, vc, a, st); break;
    case 3: launch_dec_tc<3>(q, kc, vc, a, st); break;
    case 4: launch_dec_tc<4>(q, kc, vc, a, st); break;
    case 6: launch_dec_tc<6>(q, kc, vc, a, st); break;
    case 8: launch_dec_tc<8>(q, kc, vc, a, st); break;
    default: TORCH_CHECK(false, "unsupported GQA group");
  }
}

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
    case 1: launch_tc<1>(q, kc, vc, a, B, int(max_seqlen_q), st); break;
    case 2: launch_tc<2>(q, kc, vc, a, B, int(max_seqlen_q), st); break;
    case 3: launch_tc<3>(q, kc, vc, a, B, int(max_seqlen_q), st); break;
    case 4: launch_tc<4>(q, kc, vc, a, B, int(max_seqlen_q), st); break;
    case 6: launch_tc<6>(q, kc, vc, a, B, int(max_seqlen_q), st); break;
    case 8: launch_tc<8>(q, kc, vc, a, B, int(max_seqlen_q), st); break;
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

// Device address of the error word (read by the per-step status kernel).
int64_t attn_tc_error_word_address() {
  void* p = nullptr;
  TORCH_CHECK(cudaGetSymbolAddress(&p, g_attn_tc_err) == cudaSuccess, "error word address");
  return reinterpret_cast<int64_t>(p);
}

}  // namespace isb
