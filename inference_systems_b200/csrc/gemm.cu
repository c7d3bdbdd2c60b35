// tcgen05 GEMM for sm_100a: C = A[M,K] . B[N,K]^T, bf16 inputs, fp32 accumulation in TMEM.
//
// Structure (one output tile per CTA, 192 threads):
//   warp 0      TMA producer: 128x64 "P" tile + BNx64 "Q" tile per stage into
//               128-byte-swizzled shared memory, mbarrier complete_tx.
//   warp 1      TMEM allocator + MMA issuer: 4 x tcgen05.mma (K=16) per stage,
//               tcgen05.commit releases the stage / signals the accumulator.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns per warp, fused
//               epilogue (plain store | SiLU(gate)*up | LM-head argmax with
//               Gumbel-max sampling).
// Operand roles: the 128-row MMA "M" side (P) is the activation matrix for
// large token counts and the WEIGHT matrix for <= 128 tokens (swap-AB), so a
// decode GEMM streams weights through the 128-lane tensor-core tile while the
// handful of tokens form the MMA N dimension.
// Split-K: gridDim.z CTAs of a thread-block cluster each own a K range; the
// partial accumulators are reduced through distributed shared memory by the
// cluster's rank-0 CTA (no global scratch, deterministic order).
// No TMA multicast is used anywhere in this file.

#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <vector>
#include <torch/extension.h>

#include "common.cuh"
#include "launch.cuh"

namespace isb {

// Sticky error bits of the GEMM kernels (bounded waits that gave up); 128 = the fused add+RMSNorm
// grid barrier.
__device__ unsigned int g_gemm_err;

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = BN <= 32 ? 8 : (BN <= 128 ? 6 : 4);
  static constexpr int P_BYTES = BM * BK * 2;
  static constexpr int Q_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = P_BYTES + Q_BYTES;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int RED_STRIDE = BN + 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
  static_assert(BM * RED_STRIDE * 4 + 64 * RED_STRIDE * 4 <= STAGES * STAGE_BYTES || BN > 128,
                "split-K / SiLU staging must fit in the stage buffers");
};

enum Epilogue : int { kStore = 0, kSiluMul = 1, kArgmax = 2, kRedAdd = 3, kRsPush = 4 };

struct GemmArgs {
  __nv_bfloat16* out;      // kStore / kSiluMul output
  int P_rows, Q_rows, K;
  int ldo;                 // output row stride (elements)
  int kb_per_split;
  // kArgmax
  const float* temps;      // [tokens]
  const int* rng;          // [seed, step]
  float* part_val;         // [num_vocab_tiles, tokens]
  int* part_idx;
  int vocab_offset;
  unsigned long long* dbg;  // optional per-CTA phase timestamps [ctas][8] (diagnostics)
  float* ws;                // split-K partials [tiles][splits][BM][BN] fp32
  float* acc;               // kRedAdd: fp32 accumulator [tokens][features], atomically added to
  unsigned int* counters;   // split-K arrival counters (self-resetting)
  // kRsPush (tensor-parallel reduce-scatter by token): token row t of this rank's partial product
  // belongs to rank o = t / own_rows.  Split-K CTAs first reduce into this rank's fp32 staging
  // accumulator ``acc`` (local red.add; the tile's last CTA reads the sum back and re-zeroes it);
  // the complete bf16 row is then stored into rank o's slot for this rank:
  // ``dsts[o]`` + ((rank * slot_rows + t - o * own_rows) * ldo + feature) elements.  When every
  // CTA's pushes are out, it releases ``+1`` on every rank's counter ``peer_flags[r]``.
  const unsigned long long* dsts;  // [ndst] slot-array base addresses (peer memory included)
  int ndst;
  int own_rows;                    // token rows owned by each rank
  int slot_rows;                   // rows of one source slot (>= own_rows)
  bool bcast;                      // one-shot: every row goes to every rank (slot row = token)
  const unsigned long long* peer_flags;  // [ndst] address of each rank's arrival counter
  int rank;
  // kRsPush one-shot with the residual add + RMSNorm in the same kernel (``norm_out`` set): this
  // rank's slots [ndst][slot_rows][ldo], its control words (0 arrivals, 2 arrival target of the
  // previous exchange, 4 CTA-completion counter) and the exchange error word
  const __nv_bfloat16* tp_slots;
  unsigned int* tp_ctl;
  unsigned int* tp_err;
  // kRedAdd with one K split on one rank: every accumulator element is produced by exactly one
  // CTA and the accumulator is zero between uses, so plain stores replace the atomics
  bool acc_plain;
  // kRedAdd followed, in the same kernel, by residual add + RMSNorm of the accumulated rows: after
  // a grid-wide barrier (every CTA resident: the host only asks for it when the grid fits) each CTA
  // normalises rows blockIdx, blockIdx + grid, ...: residual <- bf16(acc + residual),
  // norm_out <- RMSNorm(acc + residual), acc <- 0.  ``counters`` holds the barrier's two words.
  __nv_bfloat16* norm_out;
  __nv_bfloat16* norm_res;
  const __nv_bfloat16* norm_w;
  float norm_eps;
  bool acc_direct;         // swap-AB kRedAdd: add straight from TMEM registers (no shared staging)
  bool tma_out;            // non-swap kStore / kSiluMul / kRedAdd: stage the tile (128-byte swizzle)
                           // and leave through bulk tensor stores / reduce-adds on ``tmO``
  int epi_probe;           // diagnostics of the direct path: 1 = TMEM loads only, 2 = stores only
  int norm_rows;           // token rows of the accumulator
  bool norm_zc;
};

// Arrival counters of split-K tiles.  A launch uses one of kCounterSlots
// slices (round-robin on the host) so consecutive split-K GEMMs never share
// counters; the last CTA of a tile resets its counter to zero.
constexpr int kCounterSlots = 8;
constexpr int kCountersPerSlot = 8192;
__device__ unsigned int g_splitk_counters[kCounterSlots * kCountersPerSlot];

// Fire-and-forget reductions carry no "memory" clobber: a clobber would make the compiler reload
// every kernel argument from memory after each one (measured: a 128 x 128 fp32 tile took 6 us to
// leave the CTA instead of 1).  Readers of the reduced values are ordered by fences and barriers,
// which do clobber memory.
ISB_DEVICE void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d));
}

ISB_DEVICE void red_add_v4_sys(float* p, float a, float b, float c, float d) {
  asm volatile("red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d));
}

// Add 4 consecutive values at element offset ``off`` of the accumulator.
ISB_DEVICE void acc_add4(const GemmArgs& args, size_t off, float a, float b, float c, float d) {
  if (args.acc_plain) {
    *reinterpret_cast<float4*>(args.acc + off) = make_float4(a, b, c, d);
    return;
  }
  red_add_v4(args.acc + off, a, b, c, d);
}

ISB_DEVICE void acc_add1(const GemmArgs& args, size_t off, float a) {
  if (args.acc_plain) {
    args.acc[off] = a;
    return;
  }
  atomicAdd(args.acc + off, a);
}

// kRsPush: store 4 features of token ``tok`` (bf16) into the owner rank's slot for this rank, or
// (one-shot) into every rank's slot for this rank.
ISB_DEVICE void rs_push4(const GemmArgs& args, int tok, int f, float a, float b, float c, float d) {
  uint2 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
  h[0] = __floats2bfloat162_rn(a, b);
  h[1] = __floats2bfloat162_rn(c, d);
  if (args.bcast) {
    const size_t off = (size_t(args.rank) * args.slot_rows + tok) * args.ldo + f;
    for (int q = 0; q < args.ndst; ++q) {
      const int r = (args.rank + q) % args.ndst;  // own copy first, then the peers in turn
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(args.dsts[r]) + off) = raw;
    }
    return;
  }
  const int owner = tok / args.own_rows;
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.dsts[owner]) +
                       (size_t(args.rank) * args.slot_rows + (tok - owner * args.own_rows)) * args.ldo + f;
  *reinterpret_cast<uint2*>(dst) = raw;
}

// kRsPush: 4 features of token ``tok`` of this CTA's partial: staged (split K) or pushed.
ISB_DEVICE void rs_emit4(const GemmArgs& args, bool staged, int tok, int f, float a, float b, float c, float d) {
  if (staged) red_add_v4(args.acc + size_t(tok) * args.ldo + f, a, b, c, d);
  else rs_push4(args, tok, f, a, b, c, d);
}

// Push 4 features of token ``tok`` (bf16) into the owner rank's slot for this rank, or (one-shot)
// into every rank's slot; ``dst`` is the destination table (own slot first), the scalars are the
// kernel arguments hoisted out of the caller's loop.
ISB_DEVICE void push_rs4(const unsigned long long* dst, bool bcast, int ndst, int rk, int slot_rows, int own_rows,
                         size_t ldo, int tok, int f, float4 w) {
  uint2 raw;
  __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
  hh[0] = __floats2bfloat162_rn(w.x, w.y);
  hh[1] = __floats2bfloat162_rn(w.z, w.w);
  if (bcast) {
    const size_t off = (size_t(rk) * slot_rows + tok) * ldo + f;
    for (int q = 0; q < ndst; ++q) *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(dst[q]) + off) = raw;
  } else {
    const int owner = tok / own_rows;
    const size_t off = (size_t(rk) * slot_rows + (tok - owner * own_rows)) * ldo + f;
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(dst[(owner - rk + ndst) % ndst]) + off) = raw;
  }
}

// Byte offset of 16-byte group ``g`` (8 bf16 or 4 fp32) of row ``r`` in a non-swap output tile
// staged as boxes of 128-byte rows (128-byte swizzle), one box per ``gpb`` groups of columns.
ISB_DEVICE uint32_t nstage_off(int r, int g, int gpb) {
  return uint32_t((g / gpb) * (BM * 128) + r * 128 + (((g % gpb) ^ (r & 7)) << 4));
}

ISB_DEVICE uint32_t fmix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85EBCA6Bu;
  h ^= h >> 13;
  h *= 0xC2B2AE35u;
  h ^= h >> 16;
  return h;
}

// Counter-based uniform noise; identical to ``ops.uniform_noise`` on the host.
ISB_DEVICE float gumbel_noise(int seed, int step, int row, int col) {
  const uint32_t key = uint32_t(seed) * 0x9E3779B1u + uint32_t(step) * 0x85EBCA77u;
  uint32_t h = fmix32(uint32_t(row) * 0x27D4EB2Fu + key);
  h = fmix32(h ^ (uint32_t(col) * 0x165667B1u));
  const float u = (float(h >> 8) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

// Tail of an accumulating GEMM that also applies the residual add + RMSNorm (128 epilogue threads
// of every CTA): a bounded grid barrier, then rows round-robin over the CTAs.
__device__ __forceinline__ void fused_add_norm(const GemmArgs& args) {
  __shared__ float red[4];
  const int tid = threadIdx.x - 64;
  const unsigned int total = gridDim.x * gridDim.y * gridDim.z;
  const unsigned int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  unsigned int* arrive = args.counters;
  unsigned int* depart = args.counters + 1;
  __threadfence();
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (tid == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(arrive) : "memory");
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    for (;;) {
      unsigned int v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(arrive) : "memory");
      if (v >= total) break;
      if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicOr(&g_gemm_err, 128u);  // rows are still normalised; the step reports the error
        break;
      }
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  const int T = args.norm_rows, H = args.ldo;
  for (int row = int(cta); row < T; row += int(total)) {
    float* a = args.acc + size_t(row) * H;
    __nv_bfloat16* res = args.norm_res + size_t(row) * H;
    float ss = 0.f;
    for (int c = tid * 8; c < H; c += 128 * 8) {
      const float4 x0 = __ldcg(reinterpret_cast<const float4*>(a + c));
      const float4 x1 = __ldcg(reinterpret_cast<const float4*>(a + c + 4));
      const Vec8 r = load8(res + c);
      const float v[8] = {x0.x + r.v[0], x0.y + r.v[1], x0.z + r.v[2], x0.w + r.v[3],
                          x1.x + r.v[4], x1.y + r.v[5], x1.z + r.v[6], x1.w + r.v[7]};
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const float rs = rsqrtf((red[0] + red[1] + red[2] + red[3]) / float(H) + args.norm_eps);
    for (int c = tid * 8; c < H; c += 128 * 8) {
      const float4 x0 = __ldcg(reinterpret_cast<const float4*>(a + c));
      const float4 x1 = __ldcg(reinterpret_cast<const float4*>(a + c + 4));
      const Vec8 r = load8(res + c);
      const float v[8] = {x0.x + r.v[0], x0.y + r.v[1], x0.z + r.v[2], x0.w + r.v[3],
                          x1.x + r.v[4], x1.y + r.v[5], x1.z + r.v[6], x1.w + r.v[7]};
      store8(res + c, v);
      norm_store8(args.norm_out + size_t(row) * H + c, v, args.norm_w + c, rs, args.norm_zc);
      *reinterpret_cast<float4*>(a + c) = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(a + c + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // ``red`` is reused by the next row
  }
  if (tid == 0) {  // the last CTA out resets the barrier for the next launch on this counter slot
    unsigned int prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(depart) : "memory");
    if (prev == total - 1) {
      *arrive = 0u;
      *depart = 0u;
    }
  }
}

// Tail of a one-shot reduce-scatter GEMM that also normalises (128 epilogue threads of every CTA):
// wait (bounded) until every rank's CTAs of this exchange have counted themselves in here, then
// rows blockIdx, blockIdx + grid, ...: x = residual + sum over the source slots; residual <- bf16(x),
// norm_out <- RMSNorm(x).  The last CTA out moves the arrival target on.
__device__ __forceinline__ void rs_oneshot_norm(const GemmArgs& args) {
  __shared__ float red[4];
  __shared__ unsigned int s_target;
  const int tid = threadIdx.x - 64;
  const unsigned int total = gridDim.x * gridDim.y * gridDim.z;
  const unsigned int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  unsigned int* ctl = args.tp_ctl;
  if (tid == 0) {
    const unsigned int target = *reinterpret_cast<volatile unsigned int*>(ctl + 2) + unsigned(args.ndst) * total;
    s_target = target;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    for (;;) {
      unsigned int v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ctl) : "memory");
      if (int(v - target) >= 0) break;
      if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicOr(args.tp_err, 16u);  // rows are still normalised; the step reports the error
        break;
      }
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  const int T = args.norm_rows, H = args.ldo, W = args.ndst;
  const size_t slot_stride = size_t(args.slot_rows) * H;
  for (int row = int(cta); row < T; row += int(total)) {
    __nv_bfloat16* res = args.norm_res + size_t(row) * H;
    const __nv_bfloat16* src = args.tp_slots + size_t(row) * H;
    float x[8];
    float ss = 0.f;
    const int c = tid * 8;  // H <= 1024: one group of 8 columns per thread
    if (c < H) {
      uint4 raw[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        raw[q] = q < W ? __ldcg(reinterpret_cast<const uint4*>(src + q * slot_stride + c)) : make_uint4(0u, 0u, 0u, 0u);
      const Vec8 r = load8(res + c);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = r.v[e];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&raw[q]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(hh[e]);
          x[2 * e] += f.x;
          x[2 * e + 1] += f.y;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += x[e] * x[e];
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const float rs = rsqrtf((red[0] + red[1] + red[2] + red[3]) / float(H) + args.norm_eps);
    if (c < H) {
      store8(res + c, x);
      norm_store8(args.norm_out + size_t(row) * H + c, x, args.norm_w + c, rs, args.norm_zc);
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // ``red`` is reused by the next row
  }
  if (tid == 0) {
    unsigned int prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ctl + 4) : "memory");
    if (prev == total - 1) {
      ctl[4] = 0u;
      ctl[2] = s_target;
    }
  }
}

template <int BN, bool SWAP, int EPI, bool CL = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmO, GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + Cfg::STAGES;
  uint64_t* acc_full = empty + Cfg::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  pdl_trigger();  // the next kernel may start its own prologue now
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile_p = blockIdx.x, tile_q = blockIdx.y;
  const int kb_total = (args.K + BK - 1) / BK;
  const int kb_begin = blockIdx.z * args.kb_per_split;
  const int kb_end = min(kb_total, kb_begin + args.kb_per_split);
  const int nkb = max(kb_end - kb_begin, 0);
  const size_t cta_id = (size_t(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  unsigned long long* dbg = args.dbg ? args.dbg + cta_id * 8 : nullptr;
  if (dbg && threadIdx.x == 0) dbg[0] = globaltimer_ns();

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
    prefetch_tmap(&tmP);
    prefetch_tmap(&tmQ);
    if constexpr (SWAP && (EPI == kStore || EPI == kSiluMul || EPI == kRedAdd || EPI == kRsPush)) prefetch_tmap(&tmO);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (dbg && threadIdx.x == 0) dbg[1] = globaltimer_ns();

  if (warp == 0) {
    if (lane == 0) {
      // Weights (P under swap-AB, Q otherwise) are never written by a kernel: the
      // first STAGES weight tiles are requested before waiting for the previous
      // kernel (programmatic dependent launch), the activation tiles after it.
      auto load_w = [&](uint8_t* sp, uint64_t* bar, int kx) {
        if constexpr (SWAP) tma_load_2d(sp, &tmP, bar, kx, tile_p * BM);
        else tma_load_2d(sp + Cfg::P_BYTES, &tmQ, bar, kx, tile_q * BN);
      };
      auto load_x = [&](uint8_t* sp, uint64_t* bar, int kx) {
        if constexpr (SWAP) tma_load_2d(sp + Cfg::P_BYTES, &tmQ, bar, kx, tile_q * BN);
        else tma_load_2d(sp, &tmP, bar, kx, tile_p * BM);
      };
      const int pre = min(nkb, Cfg::STAGES);
      for (int i = 0; i < pre; ++i) {  // fresh stages: nothing to wait for
        mbar_arrive_expect_tx(&full[i], Cfg::STAGE_BYTES);
        load_w(smem + i * Cfg::STAGE_BYTES, &full[i], (kb_begin + i) * BK);
      }
      pdl_wait();
      for (int i = 0; i < nkb; ++i) {
        if (dbg && i == 0) dbg[2] = globaltimer_ns();
        const int s = i % Cfg::STAGES;
        const uint32_t ph = (i / Cfg::STAGES) & 1;
        uint8_t* sp = smem + s * Cfg::STAGE_BYTES;
        const int kx = (kb_begin + i) * BK;
        if (i >= pre) {
          if (!mbar_wait(&empty[s], ph ^ 1)) { atomicOr(&g_gemm_err, 1u); break; }
          mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
          load_w(sp, &full[s], kx);
        }
        load_x(sp, &full[s], kx);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % Cfg::STAGES;
        const uint32_t ph = (i / Cfg::STAGES) & 1;
        if (!mbar_wait(&full[s], ph)) { atomicOr(&g_gemm_err, 2u); break; }
        if (dbg && i == 0) dbg[3] = globaltimer_ns();
        tc_fence_after();
        uint8_t* sp = smem + s * Cfg::STAGE_BYTES;
        const uint64_t pd = smem_desc_sw128(sp);
        const uint64_t qd = smem_desc_sw128(sp + Cfg::P_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          // advance 16 bf16 = 32 bytes inside the swizzle atom: +2 in the >>4 address field
          mma_bf16(tmem, pd + 2 * k, qd + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      if (dbg) dbg[4] = globaltimer_ns();
      mma_commit(acc_full);
    }
  }

  // ------------------------------------------------------------ epilogue
  const bool epi = warp >= 2;
  const int quarter = warp & 3;           // TMEM lane quarter this warp may access
  const int row = quarter * 32 + lane;    // row of the P tile == TMEM lane
  const uint32_t lane_addr = tmem + (uint32_t(quarter * 32) << 16);
  const int nsplit = gridDim.z;
  const int tile_id = tile_p * gridDim.y + tile_q;
  constexpr int CH = BN < 32 ? 16 : 32;
  // shared-memory regions reused after the mainloop (every MMA has completed)
  float* xbuf = reinterpret_cast<float*>(smem);                                  // [64][RED_STRIDE]
  constexpr int XBUF_BYTES = ((64 * Cfg::RED_STRIDE * 4) + 1023) / 1024 * 1024;
  __nv_bfloat16* ostage = reinterpret_cast<__nv_bfloat16*>(smem + XBUF_BYTES);  // [BN][128] bf16
  __shared__ int s_last;

  if constexpr (CL && EPI == kRsPush) {
    // ---- split-K in ONE cluster per weight tile (cluster dims (1, 1, splits), <= 8): every CTA
    // parks its fp32 partial [tokens][features] in its own shared memory; after the cluster
    // barrier CTA r sums token rows r, r + splits, ... over the cluster (DSMEM loads) and pushes
    // them (bf16) to the owner's slot, or to every rank's slot in one-shot mode.  No staging
    // round trip through L2, no tile counter, and every CTA of the tile pushes a share.  The
    // partials stay alive until the second cluster barrier.
    static_assert(SWAP, "cluster reduce-scatter serves swap-AB tiles");
    float* fstage = reinterpret_cast<float*>(smem);  // [BN][BM] fp32 (token-major)
    __shared__ unsigned long long s_dst[8];
    const int tid = threadIdx.x - 64;
    if (epi) {
      pdl_wait();  // the slots and counters may still be in use by the previous kernel
      const bool acc_ok = mbar_wait(acc_full, 0) && nkb > 0;
      if (!acc_ok && nkb > 0) atomicOr(&g_gemm_err, 8u);
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BN / CH; ++c) {
        float v[CH];
        if (acc_ok) {
          if constexpr (CH == 16) tmem_ld16(lane_addr + c * CH, v); else tmem_ld32(lane_addr + c * CH, v);
        } else {
#pragma unroll
          for (int j = 0; j < CH; ++j) v[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < CH; ++j) fstage[(c * CH + j) * BM + row] = v[j];
      }
      if (tid < args.ndst) s_dst[tid] = args.dsts[(args.rank + tid) % args.ndst];
    }
    __syncwarp();  // .aligned cluster barrier: the warp reconverges first (lane 0 ran the pipeline)
    cluster_sync();
    if (epi) {
      const uint32_t me = cluster_ctarank(), ns = cluster_nctarank();
      const int q0 = tile_q * BN, p0 = tile_p * BM;
      const int ntok = min(BN, args.Q_rows - q0);
      const int mine = ntok > int(me) ? (ntok - int(me) + int(ns) - 1) / int(ns) : 0;  // rows of this CTA
      const bool bcast = args.bcast;
      const int ndst = args.ndst, rk = args.rank, slot_rows = args.slot_rows, own_rows = args.own_rows;
      const size_t ldo = size_t(args.ldo);
      const uint32_t base = smem_u32(fstage);
      for (int i = tid; i < mine * (BM / 4); i += 128) {
        const int t = int(me) + (i / (BM / 4)) * int(ns), f4 = (i % (BM / 4)) * 4;
        const uint32_t off = uint32_t((t * BM + f4) * 4);
        float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int z = 0; z < 8; ++z) {
          if (z < int(ns)) {
            const float4 x = ld_dsmem_f4(mapa_shared(base + off, uint32_t(z)));
            acc4.x += x.x; acc4.y += x.y; acc4.z += x.z; acc4.w += x.w;
          }
        }
        push_rs4(s_dst, bcast, ndst, rk, slot_rows, own_rows, ldo, q0 + t, p0 + f4, acc4);
      }
    }
    __syncwarp();  // .aligned cluster barrier: the warp reconverges first (lane 0 ran the pipeline)
    cluster_sync();  // the peers have finished reading this CTA's partial
  } else if constexpr (CL) {
    // ---- split-K pair in a 2-CTA cluster (swap-AB store / SiLU*mul): each CTA of the pair
    // multiplied half of K; both park their fp32 partial rows in their own shared memory, then
    // CTA r sums its own and its peer's partials (DSMEM loads) for token columns
    // [r*BN/2, (r+1)*BN/2) and runs the epilogue for that half.  The peer's partials stay
    // alive until the second cluster barrier.
    static_assert(SWAP && (EPI == kStore || EPI == kSiluMul), "cluster split-K serves swap-AB store / SiLU*mul");
    constexpr int PSTR = BN + 4;
    constexpr int HALF = BN / 2;
    constexpr int OST_BYTES = ((BN * BM * 2) + 1023) / 1024 * 1024;
    float* pbuf = reinterpret_cast<float*>(smem + XBUF_BYTES + OST_BYTES);  // [BM][PSTR]
    static_assert(XBUF_BYTES + OST_BYTES + BM * PSTR * 4 <= Cfg::STAGES * Cfg::STAGE_BYTES,
                  "cluster split-K staging must fit in the stage buffers");
    if (epi) {
      pdl_wait();
      const bool acc_ok = mbar_wait(acc_full, 0) && nkb > 0;
      if (!acc_ok && nkb > 0) atomicOr(&g_gemm_err, 8u);
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BN / CH; ++c) {
        float v[CH];
        if (acc_ok) {
          if constexpr (CH == 16) tmem_ld16(lane_addr + c * CH, v); else tmem_ld32(lane_addr + c * CH, v);
        } else {
#pragma unroll
          for (int j = 0; j < CH; ++j) v[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < CH; j += 4)
          *reinterpret_cast<float4*>(pbuf + row * PSTR + c * CH + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
    }
    __syncwarp();  // .aligned cluster barrier: the warp reconverges first (lane 0 ran the pipeline)
    cluster_sync();
    if (epi) {
      const uint32_t me = cluster_ctarank();
      const int cbase = int(me) * HALF;
      const uint32_t peer_row = mapa_shared(smem_u32(pbuf + row * PSTR + cbase), me ^ 1u);
#pragma unroll 4
      for (int j = 0; j < HALF; j += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(pbuf + row * PSTR + cbase + j);
        const float4 b4 = ld_dsmem_f4(peer_row + j * 4);
        const float sum[4] = {a4.x + b4.x, a4.y + b4.y, a4.z + b4.z, a4.w + b4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if constexpr (EPI == kStore) {
            ostage[(j + e) * BM + row] = __float2bfloat16(sum[e]);
          } else {
            if (row >= 64) xbuf[(row - 64) * Cfg::RED_STRIDE + j + e] = sum[e];
            else pbuf[row * PSTR + cbase + j + e] = sum[e];  // keep the gate sum in place
          }
        }
      }
      if constexpr (EPI == kSiluMul) {
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (row < 64) {
          for (int j = 0; j < HALF; ++j)
            ostage[j * 64 + row] =
                __float2bfloat16(silu(pbuf[row * PSTR + cbase + j]) * xbuf[row * Cfg::RED_STRIDE + j]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        const int x0 = EPI == kSiluMul ? tile_p * 64 : tile_p * BM;
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                         reinterpret_cast<uint64_t>(&tmO)),
                     "r"(x0), "r"(tile_q * BN + cbase), "r"(smem_u32(ostage))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      }
    }
    __syncwarp();  // .aligned cluster barrier: the warp reconverges first (lane 0 ran the pipeline)
    cluster_sync();  // the peer has finished reading this CTA's partials
  }
  if (epi && !CL) {
    pdl_wait();  // outputs / accumulators / split-K scratch may still be in use by the previous kernel
    bool acc_ok = mbar_wait(acc_full, 0) && nkb > 0;
    if (!acc_ok && nkb > 0) atomicOr(&g_gemm_err, 4u);
    tc_fence_after();
    if (dbg && threadIdx.x == 64) dbg[5] = globaltimer_ns();

    auto load_chunk = [&](int c, float* v) {
      if (!acc_ok || args.epi_probe == 2) {
#pragma unroll
        for (int j = 0; j < CH; ++j) v[j] = 0.f;
        return;
      }
      if constexpr (CH == 16) tmem_ld16(lane_addr + c * CH, v); else tmem_ld32(lane_addr + c * CH, v);
    };

    // ---- split-K: publish the fp32 partial to L2; the last CTA of the tile reduces
    bool reduce_here = true;
    if (nsplit > 1 && EPI != kRedAdd && EPI != kRsPush) {
      // column-major partial [BN][BM]: a warp's 32 rows of one column are 128 contiguous bytes
      float* mine = args.ws + (size_t(tile_id) * nsplit + blockIdx.z) * BN * BM + row;
      for (int c = 0; c < BN / CH; ++c) {
        float v[CH];
        load_chunk(c, v);
#pragma unroll
        for (int j = 0; j < CH; ++j) __stcg(mine + size_t(c * CH + j) * BM, v[j]);
      }
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        unsigned int* cnt = args.counters + tile_id;
        const unsigned int old = atomicAdd(cnt, 1u);
        s_last = old == unsigned(nsplit - 1);
        if (s_last) *cnt = 0u;  // every split has arrived: reset for the next launch
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      reduce_here = s_last != 0;
      if (reduce_here) __threadfence();
    }

    if (reduce_here) {
      const int p0 = tile_p * BM, q0 = tile_q * BN;
      for (int c = 0; c < BN / CH; ++c) {
        if constexpr (EPI == kSiluMul && !SWAP) {
          if ((c * CH) % 128 >= 64) continue;  // up chunks are consumed with their gate chunk
        }
        float v[CH];
        load_chunk(c, v);
        auto add_partials = [&](float* acc, int col0) {
          for (int z = 0; z < nsplit; ++z) {
            if (z == int(blockIdx.z)) continue;
            const float* src = args.ws + (size_t(tile_id) * nsplit + z) * BN * BM + size_t(col0) * BM + row;
#pragma unroll
            for (int j = 0; j < CH; ++j) acc[j] += __ldcg(src + size_t(j) * BM);
          }
        };
        if (nsplit > 1 && EPI != kRedAdd && EPI != kRsPush) add_partials(v, c * CH);
        if constexpr (EPI == kStore) {
          if constexpr (SWAP) {
            // transpose through shared memory: ostage[token][feature]
#pragma unroll
            for (int j = 0; j < CH; ++j) ostage[(c * CH + j) * BM + row] = __float2bfloat16(v[j]);
          } else if (args.tma_out) {
            // 8 bf16 per 16-byte group; 64-column boxes (8 groups)
#pragma unroll
            for (int j = 0; j < CH / 8; ++j) {
              uint4 pk;
              __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
              for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
              *reinterpret_cast<uint4*>(smem + nstage_off(row, (c * CH) / 8 + j, 8)) = pk;
            }
          } else {
            const int t = p0 + row;
            const int col0 = q0 + c * CH;
            if (t < args.P_rows) {
              __nv_bfloat16* o = args.out + size_t(t) * args.ldo + col0;
              if (col0 + CH <= args.Q_rows && (args.ldo % 8) == 0) {
#pragma unroll
                for (int j = 0; j < CH / 8; ++j) {
                  uint4 pk;
                  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                  for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
                  reinterpret_cast<uint4*>(o)[j] = pk;
                }
              } else {
#pragma unroll
                for (int j = 0; j < CH; ++j)
                  if (col0 + j < args.Q_rows) o[j] = __float2bfloat16(v[j]);
              }
            }
          }
        } else if constexpr (EPI == kSiluMul) {
          if constexpr (SWAP) {
            // gate rows 0..63, up rows 64..127 of this weight tile
            if (row >= 64) {
#pragma unroll
              for (int j = 0; j < CH; ++j) xbuf[(row - 64) * Cfg::RED_STRIDE + c * CH + j] = v[j];
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (row < 64) {
#pragma unroll
              for (int j = 0; j < CH; ++j) {
                const float u = xbuf[row * Cfg::RED_STRIDE + c * CH + j];
                ostage[(c * CH + j) * 64 + row] = __float2bfloat16(silu(v[j]) * u);
              }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
          } else {
            float u[CH];
            load_chunk(c + 64 / CH, u);
            if (nsplit > 1) add_partials(u, c * CH + 64);
            const int t = p0 + row;
            const int within = (c * CH) % 128;
            const int g = (c * CH) / 128;
            const int col0 = q0 / 2 + g * 64 + within;
            if (args.tma_out) {  // output column (within the tile) g * 64 + within + j
#pragma unroll
              for (int j = 0; j < CH / 8; ++j) {
                uint4 pk;
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  h[e] = __floats2bfloat162_rn(silu(v[8 * j + 2 * e]) * u[8 * j + 2 * e],
                                               silu(v[8 * j + 2 * e + 1]) * u[8 * j + 2 * e + 1]);
                *reinterpret_cast<uint4*>(smem + nstage_off(row, (g * 64 + within) / 8 + j, 8)) = pk;
              }
            } else if (t < args.P_rows) {
#pragma unroll
              for (int j = 0; j < CH; ++j)
                if (col0 + j < args.Q_rows / 2)
                  args.out[size_t(t) * args.ldo + col0 + j] = __float2bfloat16(silu(v[j]) * u[j]);
            }
          }
        } else if constexpr (EPI == kRsPush) {
          if constexpr (SWAP) {
            float* fstage = reinterpret_cast<float*>(smem);  // [BN][BM] fp32 (token-major)
#pragma unroll
            for (int j = 0; j < CH; ++j) fstage[(c * CH + j) * BM + row] = v[j];
          } else {
            const int t = p0 + row;
            const int col0 = q0 + c * CH;
            if (t < args.P_rows) {
#pragma unroll
              for (int j = 0; j < CH / 4; ++j)
                if (col0 + 4 * j < args.Q_rows)
                  rs_emit4(args, nsplit > 1, t, col0 + 4 * j, v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
          }
        } else if constexpr (EPI == kRedAdd) {
          if constexpr (SWAP) {
            if (args.acc_direct) {
              // thread = feature row, v[j] = token c*CH + j: a warp adds 32 consecutive features
              const int f = p0 + row;
              if (args.epi_probe == 1) {
                float sink = 0.f;
#pragma unroll
                for (int j = 0; j < CH; ++j) sink += v[j];
                if (sink == 123.456f) args.acc[0] = sink;  // keeps the loads
              } else if (f < args.P_rows) {
                // conditions hoisted out of the store loop: full chunks store unpredicated
                const size_t ldo = size_t(args.ldo);
                float* dst = args.acc + size_t(q0 + c * CH) * ldo + f;
                const int nj = min(CH, args.Q_rows - (q0 + c * CH));
                const int reps = args.epi_probe == 3 ? 17 : 1;  // diagnostics: repeated stores
                for (int rr = 0; rr < reps; ++rr) {
                  if (args.acc_plain && nj == CH) {
#pragma unroll
                    for (int j = 0; j < CH; ++j) dst[j * ldo] = v[j];
                  } else if (nj == CH) {
#pragma unroll
                    for (int j = 0; j < CH; ++j)
                      asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(dst + j * ldo), "f"(v[j]));
                  } else {
                    for (int j = 0; j < nj; ++j) {
                      if (args.acc_plain) dst[j * ldo] = v[j];
                      else asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(dst + j * ldo), "f"(v[j]));
                    }
                  }
                }
              }
            } else {
              float* fstage = reinterpret_cast<float*>(smem);  // [BN][BM] fp32 (token-major)
#pragma unroll
              for (int j = 0; j < CH; ++j) fstage[(c * CH + j) * BM + row] = v[j];
            }
          } else if (args.tma_out) {  // 4 fp32 per 16-byte group; 32-column boxes (8 groups)
#pragma unroll
            for (int j = 0; j < CH / 4; ++j)
              *reinterpret_cast<float4*>(smem + nstage_off(row, (c * CH) / 4 + j, 8)) =
                  make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          } else {
            const int t = p0 + row;
            const int col0 = q0 + c * CH;
            if (t < args.P_rows) {
              const size_t off = size_t(t) * args.ldo + col0;
              if (col0 + CH <= args.Q_rows && (args.ldo % 4) == 0) {
#pragma unroll
                for (int j = 0; j < CH / 4; ++j) acc_add4(args, off + 4 * j, v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
              } else {
#pragma unroll
                for (int j = 0; j < CH; ++j)
                  if (col0 + j < args.Q_rows) acc_add1(args, off + j, v[j]);
              }
            }
          }
        } else {  // kArgmax: LM head fused with greedy / Gumbel-max selection
          const int seed = args.rng[0], step = args.rng[1];
          if constexpr (SWAP) {
            // rows = vocab entries, columns = tokens.  Scores go to shared memory
            // ([row][col], stride BN+1: conflict-free both ways) and one thread per
            // token column scans the 128 rows, keeping the first maximum.
            float* sc_s = xbuf;                                   // [BM][BN + 1]
            float* temp_s = xbuf + BM * (BN + 1);                 // [BN]
            if (c == 0) {
              for (int j = threadIdx.x - 64; j < BN; j += 128) temp_s[j] = q0 + j < args.Q_rows ? args.temps[q0 + j] : 0.f;
              asm volatile("bar.sync 1, 128;" ::: "memory");
            }
            const int vrow = p0 + row;
            const bool valid = vrow < args.P_rows;
#pragma unroll
            for (int j = 0; j < CH; ++j) {
              const int col = c * CH + j;
              float sc = valid ? v[j] : -INFINITY;
              const float temp = temp_s[col];
              if (valid && temp > 1e-10f) sc = sc / temp + gumbel_noise(seed, step, q0 + col, args.vocab_offset + vrow);
              sc_s[row * (BN + 1) + col] = sc;
            }
            if (c == BN / CH - 1) {
              asm volatile("bar.sync 1, 128;" ::: "memory");
              for (int col = threadIdx.x - 64; col < BN; col += 128) {
                const int t = q0 + col;
                float best = -INFINITY;
                int bi = 0;
                for (int r = 0; r < BM; ++r) {
                  const float x = sc_s[r * (BN + 1) + col];
                  if (x > best) { best = x; bi = r; }
                }
                if (t < args.Q_rows) {
                  args.part_val[size_t(tile_p) * args.Q_rows + t] = best;
                  args.part_idx[size_t(tile_p) * args.Q_rows + t] = p0 + bi;
                }
              }
            }
          } else {
            const int t = p0 + row;
            if (t < args.P_rows) {
              const float temp = args.temps[t];
              float best = -INFINITY;
              int bi = 0x7fffffff;
#pragma unroll
              for (int j = 0; j < CH; ++j) {
                const int vcol = q0 + c * CH + j;
                if (vcol < args.Q_rows) {
                  float sc = v[j];
                  if (temp > 1e-10f) sc = sc / temp + gumbel_noise(seed, step, t, args.vocab_offset + vcol);
                  if (sc > best) { best = sc; bi = vcol; }
                }
              }
              const size_t slot = size_t(tile_q) * args.P_rows + t;
              if (c == 0 || best > args.part_val[slot] || (best == args.part_val[slot] && bi < args.part_idx[slot])) {
                args.part_val[slot] = best;
                args.part_idx[slot] = bi;
              }
            }
          }
        }
      }
      // non-swap staged tiles leave through bulk tensor stores (reduce-adds for the accumulator),
      // one per 128-byte-wide box; the copy engine clips rows and columns past the output
      if constexpr (!SWAP && (EPI == kStore || EPI == kSiluMul || EPI == kRedAdd)) {
        if (args.tma_out) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (threadIdx.x == 64) {
            const uint64_t map = reinterpret_cast<uint64_t>(&tmO);
            constexpr int NBOX = EPI == kRedAdd ? BN / 32 : EPI == kSiluMul ? BN / 128 : BN / 64;
            constexpr int BOXC = EPI == kRedAdd ? 32 : 64;  // columns per box
            const int c0 = EPI == kSiluMul ? q0 / 2 : q0;
#pragma unroll
            for (int bx = 0; bx < NBOX; ++bx) {
              const uint32_t src = smem_u32(smem + bx * (BM * 128));
              if (EPI == kRedAdd && !args.acc_plain)
                asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];"
                             ::"l"(map), "r"(c0 + bx * BOXC), "r"(p0), "r"(src) : "memory");
              else
                asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                             ::"l"(map), "r"(c0 + bx * BOXC), "r"(p0), "r"(src) : "memory");
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            if (EPI == kRedAdd && args.norm_out != nullptr) {
              asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
              asm volatile("fence.proxy.async.global;" ::: "memory");
            } else {
              asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            }
          }
        }
      }
      // swap-AB accumulation: the staged [tokens][features] fp32 tile leaves in ONE bulk tensor
      // reduce-add (a plain bulk store when this CTA is the tile's only producer); the copy
      // engine clips token rows past the accumulator's extent
      if (SWAP && EPI == kRedAdd && !args.acc_direct) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const uint64_t map = reinterpret_cast<uint64_t>(&tmO);
          if (args.acc_plain)
            asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map),
                         "r"(p0), "r"(q0), "r"(smem_u32(smem))
                         : "memory");
          else
            asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map),
                         "r"(p0), "r"(q0), "r"(smem_u32(smem))
                         : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          // the fused norm tail reads the sums in this kernel: wait for the writes themselves
          // and order them (async proxy) before this CTA's generic release; otherwise only the
          // shared-memory source must stay intact until the copy has read it
          if (args.norm_out != nullptr) {
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
            asm volatile("fence.proxy.async.global;" ::: "memory");
          } else {
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          }
        }
      }
      if constexpr (EPI == kRsPush) {
        const int tid = threadIdx.x - 64;
        // Destination table in shared memory (own slot first, then the peers in turn), read once;
        // every loop below stores without per-element branches on kernel arguments (a branch per
        // store cut this epilogue's store rate by a factor of five).
        __shared__ unsigned long long s_dst[8];
        const int ndst = args.ndst, rk = args.rank;
        const bool bcast = args.bcast;
        const size_t ldo = size_t(args.ldo);
        if (tid < ndst) s_dst[tid] = args.dsts[(rk + tid) % ndst];
        asm volatile("bar.sync 1, 128;" ::: "memory");
        auto push4 = [&](int tok, int f, float4 w) {
          uint2 raw;
          __nv_bfloat162* hh = reinterpret_cast<__nv_bfloat162*>(&raw);
          hh[0] = __floats2bfloat162_rn(w.x, w.y);
          hh[1] = __floats2bfloat162_rn(w.z, w.w);
          if (bcast) {
            const size_t off = (size_t(rk) * args.slot_rows + tok) * ldo + f;
            for (int q = 0; q < ndst; ++q) *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(s_dst[q]) + off) = raw;
          } else {
            const int owner = tok / args.own_rows;
            const size_t off = (size_t(rk) * args.slot_rows + (tok - owner * args.own_rows)) * ldo + f;
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(s_dst[(owner - rk + ndst) % ndst]) + off) = raw;
          }
        };
        if constexpr (SWAP) {
          const float* fstage = reinterpret_cast<const float*>(smem);
          const int ntok = min(BN, args.Q_rows - q0);  // feature rows are whole tiles (N % 128 == 0)
          if (nsplit > 1) {
            // split-K partials meet in the local fp32 staging rows through one bulk tensor
            // reduce-add per CTA (the copy engine clips rows past the tokens)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (threadIdx.x == 64) {
              asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];"
                           ::"l"(reinterpret_cast<uint64_t>(&tmO)), "r"(p0), "r"(q0), "r"(smem_u32(smem))
                           : "memory");
              asm volatile("cp.async.bulk.commit_group;" ::: "memory");
              asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
              asm volatile("fence.proxy.async.global;" ::: "memory");
            }
          } else {
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the staged tile is complete
            for (int i = tid; i < ntok * (BM / 4); i += 128) {
              const int t = i / (BM / 4), f4 = (i % (BM / 4)) * 4;
              push4(q0 + t, p0 + f4, *reinterpret_cast<const float4*>(fstage + t * BM + f4));
            }
          }
        }
        if (nsplit > 1) {
          // the tile's last split reads the reduced partial back, re-zeroes it and pushes it
          __threadfence();
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (threadIdx.x == 64) {
            unsigned int* cnt = args.counters + tile_id;
            const unsigned int old = atomicAdd(cnt, 1u);
            s_last = old == unsigned(nsplit - 1);
            if (s_last) *cnt = 0u;
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (s_last) {
            __threadfence();
            const int tok0 = SWAP ? q0 : p0, ntok = SWAP ? BN : BM;
            const int f0 = SWAP ? p0 : q0, nf = SWAP ? BM : BN;
            const int T = SWAP ? args.Q_rows : args.P_rows, F = SWAP ? args.P_rows : args.Q_rows;
            // 8 independent L2 reads in flight per thread before any store
            constexpr int UN = 8;
            const int total = min(ntok, T - tok0) * (nf / 4);
            for (int base = tid; base < total; base += 128 * UN) {
              float4 w[UN];
#pragma unroll
              for (int u = 0; u < UN; ++u) {
                const int i = min(base + u * 128, total - 1);
                const int tok = tok0 + i / (nf / 4), f = f0 + (i % (nf / 4)) * 4;
                w[u] = f < F ? __ldcg(reinterpret_cast<const float4*>(args.acc + size_t(tok) * ldo + f))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int u = 0; u < UN; ++u) {
                const int i = base + u * 128;
                if (i >= total) break;
                const int tok = tok0 + i / (nf / 4), f = f0 + (i % (nf / 4)) * 4;
                if (f >= F) continue;
                *reinterpret_cast<float4*>(args.acc + size_t(tok) * ldo + f) = make_float4(0.f, 0.f, 0.f, 0.f);
                push4(tok, f, w[u]);
              }
            }
          }
        }
      }
      // swap-AB stores leave through one TMA tensor store of the staged tile
      if constexpr (SWAP && (EPI == kStore || EPI == kSiluMul)) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const int x0 = EPI == kSiluMul ? tile_p * 64 : tile_p * BM;
          asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                           reinterpret_cast<uint64_t>(&tmO)),
                       "r"(x0), "r"(q0), "r"(smem_u32(ostage))
                       : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        }
      }
    }
  }
  if (dbg && threadIdx.x == 64) dbg[6] = globaltimer_ns();
  if constexpr (EPI == kRedAdd) {
    if (args.norm_out != nullptr && epi) fused_add_norm(args);
  }
  if constexpr (EPI == kRsPush) {
    // Every CTA counts itself in on every rank once its pushes are issued: one system-scope fence
    // by one thread after the epilogue barrier orders all 128 epilogue threads' stores (and, for
    // the tile's last split, the staged sums it read) before the counts; the owners wait for
    // world x gridDim CTAs.  No fence drains the whole grid; only the fused one-shot norm makes a
    // CTA wait for the other ranks' CTAs (bounded).
    if (epi) {
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");  // one fence orders the stores before every count
        for (int r = 0; r < args.ndst; ++r) {
          unsigned int* flag = reinterpret_cast<unsigned int*>(args.peer_flags[(args.rank + r) % args.ndst]);
          asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(flag) : "memory");
        }
      }
      if (args.norm_out != nullptr) rs_oneshot_norm(args);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
  if (dbg && threadIdx.x == 0) dbg[7] = globaltimer_ns();
}

// Persistent LM head (swap-AB: vocabulary rows are the 128-row MMA side, the <= 128 tokens the
// N side): one CTA per SM walks vocabulary tiles with a stride of gridDim.x.  Two TMEM
// accumulators alternate, so while the epilogue warps reduce tile i to per-token
// (max, argmax) through shared memory, the producer and MMA warps already stream and multiply
// tile i+1.  The per-tile results go to the same [tiles][tokens] partials as the one-tile-per-CTA
// path and the same second-stage kernel finishes the selection.
ISB_DEVICE void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

static int num_sms();

template <int BN>
struct LmCfg {
  static constexpr int CH = BN < 32 ? 16 : 32;  // score columns staged and scanned at a time
  static constexpr int P_BYTES = BM * BK * 2;
  static constexpr int Q_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = P_BYTES + Q_BYTES;
  static constexpr int SC_BYTES = 2 * BM * (CH + 1) * 4;  // one staging slice per epilogue warpgroup
  static constexpr int STAGES = (220 * 1024 - SC_BYTES - BN * 4) / STAGE_BYTES < 8
                                    ? (220 * 1024 - SC_BYTES - BN * 4) / STAGE_BYTES : 8;
  static constexpr int ACC_COLS = BN < 32 ? 32 : BN;
  static constexpr int TMEM_COLS = 2 * ACC_COLS < 64 ? 64 : 2 * ACC_COLS;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + SC_BYTES + BN * 4 + 256;
};

constexpr int kLmThreads = 320;  // producer warp, MMA warp, two epilogue warpgroups

template <int BN>
__global__ void __launch_bounds__(kLmThreads, 1)
    lm_head_persistent_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                              GemmArgs args, int ntiles) {
  using Cfg = LmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sc_all = reinterpret_cast<float*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);  // [2][BM][CH + 1]
  float* temp_s = sc_all + 2 * BM * (Cfg::CH + 1);                                 // [BN]
  uint64_t* full = reinterpret_cast<uint64_t*>(temp_s + BN);
  uint64_t* empty = full + Cfg::STAGES;
  uint64_t* acc_full = empty + Cfg::STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb_total = (args.K + BK - 1) / BK;
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 256);
    }
    fence_mbar_init();
    prefetch_tmap(&tmP);
    prefetch_tmap(&tmQ);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int i = 0;
      for (int lt = 0; lt < my_tiles; ++lt) {
        const int tile = blockIdx.x + lt * gridDim.x;
        for (int kb = 0; kb < kb_total; ++kb, ++i) {
          const int s = i % Cfg::STAGES;
          if (i >= Cfg::STAGES && !mbar_wait(&empty[s], ((i / Cfg::STAGES) & 1) ^ 1)) {
            atomicOr(&g_gemm_err, 16u);
            lt = my_tiles;
            break;
          }
          uint8_t* sp = smem + s * Cfg::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
          tma_load_2d(sp, &tmP, &full[s], kb * BK, tile * BM);
          tma_load_2d(sp + Cfg::P_BYTES, &tmQ, &full[s], kb * BK, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int i = 0;
      bool ok = true;
      for (int lt = 0; ok && lt < my_tiles; ++lt) {
        const int buf = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt >> 1) - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc = tmem + buf * Cfg::ACC_COLS;
        for (int kb = 0; kb < kb_total; ++kb, ++i) {
          const int s = i % Cfg::STAGES;
          if (!mbar_wait(&full[s], (i / Cfg::STAGES) & 1)) { ok = false; break; }
          tc_fence_after();
          uint8_t* sp = smem + s * Cfg::STAGE_BYTES;
          const uint64_t pd = smem_desc_sw128(sp), qd = smem_desc_sw128(sp + Cfg::P_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) mma_bf16(acc, pd + 2 * k, qd + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        mma_commit(&acc_full[buf]);
      }
      if (!ok) atomicOr(&g_gemm_err, 32u);
    }
  } else {
    // ---- epilogue: warpgroups of warps 2..5 and 6..9; TMEM lane quarter = warp % 4; warpgroup eh
    // owns the column chunks c with c % 2 == eh
    const int eh = (warp - 2) >> 2;
    const int et = (threadIdx.x - 64) & 127;  // thread index inside the warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;      // vocabulary row within the tile == TMEM lane
    const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
    constexpr int CH = Cfg::CH;
    constexpr int NCH = BN / CH;
    float* sc_s = sc_all + eh * BM * (CH + 1);
    const int seed = args.rng[0], step = args.rng[1];
    for (int j = threadIdx.x - 64; j < BN; j += 256) temp_s[j] = j < args.Q_rows ? args.temps[j] : 0.f;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    bool ok = true;
    for (int lt = 0; lt < my_tiles; ++lt) {
      const int tile = blockIdx.x + lt * gridDim.x;
      const int buf = lt & 1;
      if (!mbar_wait(&acc_full[buf], (lt >> 1) & 1)) ok = false;
      tc_fence_after();
      const int vrow = tile * BM + row;
      const bool valid = ok && vrow < args.P_rows;
      const int my_last = NCH - 1 - ((NCH - 1 - eh) & 1);  // last chunk of this warpgroup (may be < 0)
      if (my_last < 0) {
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
      }
#pragma unroll 1
      for (int c = eh; c < NCH; c += 2) {
        float v[CH];
        const uint32_t taddr = tmem + buf * Cfg::ACC_COLS + lane_addr + c * CH;
        if constexpr (CH == 16) tmem_ld16(taddr, v); else tmem_ld32(taddr, v);
        if (c == my_last) {
          tc_fence_before();
          mbar_arrive(&acc_empty[buf]);  // this warpgroup has read all its columns of the accumulator
        }
#pragma unroll
        for (int x = 0; x < CH; ++x) {
          const int col = c * CH + x;
          float sc = valid ? v[x] : -INFINITY;
          const float temp = temp_s[col];
          if (valid && temp > 1e-10f) sc = sc / temp + gumbel_noise(seed, step, col, args.vocab_offset + vrow);
          sc_s[row * (CH + 1) + x] = sc;
        }
        named_bar_sync(2 + eh, 128);
        // CH columns, 128 / CH threads per column, each scanning a slice of the rows
        constexpr int TPC = 128 / CH, RPT = BM / TPC;
        const int x = et % CH, part = et / CH;
        float best = -INFINITY;
        int bi = 0;
        for (int r = part * RPT; r < (part + 1) * RPT; ++r) {
          const float y = sc_s[r * (CH + 1) + x];
          if (y > best) { best = y; bi = r; }
        }
#pragma unroll
        for (int o = CH; o < 32; o <<= 1) {  // combine the row slices held by lanes CH, 2CH, .. apart
          const float ob = __shfl_xor_sync(0xffffffffu, best, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        float* red_v = reinterpret_cast<float*>(sc_s);  // reuse after the scan: [4 warps][CH]
        named_bar_sync(2 + eh, 128);
        if ((et & 31) < CH) {
          red_v[(et >> 5) * CH + x] = best;
          reinterpret_cast<int*>(red_v + 4 * CH)[(et >> 5) * CH + x] = bi;
        }
        named_bar_sync(2 + eh, 128);
        if (et < CH) {
          float b2 = red_v[x];
          int i2 = reinterpret_cast<int*>(red_v + 4 * CH)[x];
          for (int w = 1; w < 4; ++w) {
            const float ob = red_v[w * CH + x];
            const int oi = reinterpret_cast<int*>(red_v + 4 * CH)[w * CH + x];
            if (ob > b2 || (ob == b2 && oi < i2)) { b2 = ob; i2 = oi; }
          }
          const int col = c * CH + x;
          if (col < args.Q_rows) {
            args.part_val[size_t(tile) * args.Q_rows + col] = b2;
            args.part_idx[size_t(tile) * args.Q_rows + col] = tile * BM + i2;
          }
        }
        named_bar_sync(2 + eh, 128);  // sc_s is rewritten by the next chunk / tile
      }
    }
    if (!ok) atomicOr(&g_gemm_err, 64u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

template <int BN>
static void launch_lm_persistent(const CUtensorMap& tp, const CUtensorMap& tq, const GemmArgs& a, int tiles,
                                 cudaStream_t st) {
  using Cfg = LmCfg<BN>;
  auto kern = lm_head_persistent_kernel<BN>;
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) == cudaSuccess,
                "persistent LM head smem attribute");
    attr = true;
  }
  const int grid = std::min(tiles, num_sms());
  launch_pdl(kern, dim3(grid), dim3(kLmThreads), Cfg::SMEM, st, tp, tq, a, tiles);
}

// Second stage of the fused LM-head selection: best (score, index) over vocab tiles.
__global__ void argmax_tiles_kernel(const float* __restrict__ pv, const int* __restrict__ pi, int ntiles, int tokens,
                                    int vocab_offset, float* __restrict__ out_val, int* __restrict__ out_idx) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < ntiles; i += blockDim.x) {
    const float s = pv[size_t(i) * tokens + t];
    const int ix = pi[size_t(i) * tokens + t];
    if (s > best || (s == best && ix < bi)) { best = s; bi = ix; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float os = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (os > best || (os == best && oi < bi)) { best = os; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x >> 5); ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
    out_val[t] = best;
    out_idx[t] = bi + vocab_offset;
  }
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
                    q == cudaDriverEntryPointSuccess && p,
                "cannot resolve cuTensorMapEncodeTiled");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 K-major map: dims {K, rows}, box {64, box_rows}, 128-byte swizzle, zero OOB fill.
static CUtensorMapL2promotion promo_mode() {
  static int mode = -1;
  if (mode < 0) {
    const char* e = std::getenv("ISB_TMA_PROMO");
    mode = e ? std::atoi(e) : 3;
  }
  return mode == 0 ? CU_TENSOR_MAP_L2_PROMOTION_NONE
                   : mode == 1 ? CU_TENSOR_MAP_L2_PROMOTION_L2_64B
                               : mode == 2 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B : CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
}

CUtensorMap make_kmajor_map(const void* ptr, int64_t rows, int64_t K, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(K) * 2};
  cuuint32_t box[2] = {cuuint32_t(BK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo_mode(),
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", int(r));
  return m;
}

// Cluster split-K pair (swap-AB store / SiLU*mul): grid (tiles_p, tiles_q, 2), cluster (1, 1, 2).
template <int BN, int EPI>
static void launch_gemm_pair(const CUtensorMap& tp, const CUtensorMap& tq, const CUtensorMap& to, GemmArgs a,
                             int tiles_p, int tiles_q, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_tc_kernel<BN, true, EPI, true>;
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) == cudaSuccess);
    attr = true;
  }
  launch_pdl_cluster(kern, dim3(tiles_p, tiles_q, 2), dim3(kThreads), Cfg::SMEM, stream, dim3(1, 1, 2), tp, tq, to, a);
  const cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, "gemm (cluster pair) launch failed: ", cudaGetErrorString(e));
}

// Reduce-scatter GEMM with the K splits of each weight tile in one thread-block cluster.
template <int BN>
static void launch_rs_cluster(const CUtensorMap& tp, const CUtensorMap& tq, GemmArgs a, int tiles_p, int tiles_q,
                              int splits, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_tc_kernel<BN, true, kRsPush, true>;
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) == cudaSuccess);
    attr = true;
  }
  launch_pdl_cluster(kern, dim3(tiles_p, tiles_q, splits), dim3(kThreads), Cfg::SMEM, stream, dim3(1, 1, splits), tp, tq,
                     tp, a);
  const cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, "gemm (reduce-scatter cluster) launch failed: ", cudaGetErrorString(e));
}

static bool gemm_pair_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("ISB_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int BN, bool SWAP, int EPI>
static void launch_gemm(const CUtensorMap& tp, const CUtensorMap& tq, const CUtensorMap& to, GemmArgs a, int tiles_p,
                        int tiles_q, int splits, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_tc_kernel<BN, SWAP, EPI>;
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) == cudaSuccess);
    attr = true;
  }
  launch_pdl(kern, dim3(tiles_p, tiles_q, splits), dim3(kThreads), Cfg::SMEM, stream, tp, tq, to, a);
  const cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, "gemm launch failed: ", cudaGetErrorString(e));
}

// 2-D bf16 row-major output map for the swap-AB TMA store: dims {cols, rows}, box {box_cols, box_rows}.
static CUtensorMap make_store_map(const void* ptr, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
  cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (store) failed: ", int(r));
  return m;
}

// 2-D fp32 row-major accumulator map for the swap-AB TMA reduce-add: dims {cols, rows}, box
// {box_cols, box_rows}; rows past ``rows`` are clipped by the copy.
static CUtensorMap make_acc_map(const void* ptr, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols) * 4};
  cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (accumulator) failed: ", int(r));
  return m;
}

// Output map of a non-swap tile staged in 128-byte-swizzled boxes of [128 rows x 128 bytes]:
// bf16 (``fp32`` false, 64 columns per box) or fp32 (32 columns per box); dims {cols, rows}.
static CUtensorMap make_out_map_sw128(const void* ptr, int64_t rows, int64_t cols, bool fp32) {
  CUtensorMap m;
  const int es = fp32 ? 4 : 2;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols) * es};
  cuuint32_t box[2] = {cuuint32_t(128 / es), cuuint32_t(BM)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                           const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (swizzled output) failed: ", int(r));
  return m;
}

// Non-swap tiles leave through bulk tensor copies when the output rows are 16-byte multiples.
static bool out_map_ok(const void* ptr, int64_t cols, bool fp32) {
  static const bool on = [] {
    const char* e = std::getenv("ISB_GEMM_TMA_OUT");
    return !(e && e[0] == '0');
  }();
  return on && (cols * (fp32 ? 4 : 2)) % 16 == 0 && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// ISB_GEMM_SWAP_HALVE=0 keeps one token tile per weight tile for 65..128 tokens.
static bool swap_halve_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("ISB_GEMM_SWAP_HALVE");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Token tile of a swap-AB GEMM.  For the store and SiLU-mul GEMMs with 65..128 tokens and fewer
// than half as many weight tiles as SMs, two 64-token tiles per weight tile put twice as many SMs
// to work (the tensor-core time of one 128-token tile, not the weight stream, bounds such a CTA;
// the second read of a weight tile mostly hits L2): gate_up + SiLU at 128 tokens 16.2 -> 12.1 us,
// qkv 8.2 -> 7.6 us.  The split-K accumulating GEMMs keep 128-token tiles (halving them costs
// K splits: down 10.2 -> 13.1 us).
static int pick_bn_swap(int tokens, int weight_tiles = 0) {  // 0: keep one token tile
  if (tokens <= 16) return 16;
  if (tokens <= 32) return 32;
  if (tokens <= 64) return 64;
  if (swap_halve_enabled() && weight_tiles > 0 && 2 * weight_tiles <= num_sms()) return 64;
  return 128;
}

// Split-K factor: grow while the grid stays within ~1.5 waves and every split keeps >= 2 k-blocks.
static int pick_splits(int tiles, int kb_total, int max_split = 8) {
  int s = 1;
  const int sms = num_sms();
  while (s < max_split && tiles * (s * 2) <= 2 * sms && kb_total / (s * 2) >= 2) s *= 2;
  return s;
}

static unsigned int* counter_slot() {
  static unsigned int* base[64] = {};
  static unsigned int next = 0;
  int dev;
  cudaGetDevice(&dev);
  if (!base[dev]) {
    void* p = nullptr;
    TORCH_CHECK(cudaGetSymbolAddress(&p, g_splitk_counters) == cudaSuccess, "split-K counters unavailable");
    base[dev] = static_cast<unsigned int*>(p);
  }
  return base[dev] + (next++ % kCounterSlots) * kCountersPerSlot;
}

template <int EPI, bool SWAP>
static void dispatch_bn(int bn, const CUtensorMap& tp, const CUtensorMap& tq, const CUtensorMap& to, GemmArgs a,
                        int tp_, int tq_, int s, cudaStream_t st) {
  switch (bn) {
    case 16: launch_gemm<16, SWAP, EPI>(tp, tq, to, a, tp_, tq_, s, st); break;
    case 32: launch_gemm<32, SWAP, EPI>(tp, tq, to, a, tp_, tq_, s, st); break;
    case 64: launch_gemm<64, SWAP, EPI>(tp, tq, to, a, tp_, tq_, s, st); break;
    case 128: launch_gemm<128, SWAP, EPI>(tp, tq, to, a, tp_, tq_, s, st); break;
    default: TORCH_CHECK(false, "unsupported tile width");
  }
}

struct Plan {
  bool swap;
  int bn, tiles_p, tiles_q, splits, kb_per;
  CUtensorMap tp, tq;
};

static Plan plan_gemm(const at::Tensor& a, const at::Tensor& b, bool allow_split, int force_splits = 0,
                      bool halve_tokens = false) {
  const int M = a.size(0), K = a.size(1), N = b.size(0);
  Plan p;
  p.swap = M <= 128;
  const int kb_total = (K + BK - 1) / BK;
  if (p.swap) {
    p.tiles_p = (N + BM - 1) / BM;
    p.bn = halve_tokens ? pick_bn_swap(M, p.tiles_p) : pick_bn_swap(M);
    p.tiles_q = (M + p.bn - 1) / p.bn;
    p.tp = make_kmajor_map(b.data_ptr(), N, K, BM);
    p.tq = make_kmajor_map(a.data_ptr(), M, K, p.bn);
  } else {
    p.bn = 256;
    p.tiles_p = (M + BM - 1) / BM;
    p.tiles_q = (N + 255) / 256;
    p.tp = make_kmajor_map(a.data_ptr(), M, K, BM);
    p.tq = make_kmajor_map(b.data_ptr(), N, K, 256);
  }
  int s = allow_split ? pick_splits(p.tiles_p * p.tiles_q, kb_total) : 1;
  if (force_splits > 0) s = std::min(force_splits, kb_total);
  p.kb_per = (kb_total + s - 1) / s;
  p.splits = (kb_total + p.kb_per - 1) / p.kb_per;
  TORCH_CHECK(p.tiles_p * p.tiles_q <= kCountersPerSlot || p.splits == 1, "too many split-K tiles");
  return p;
}

static void check_operands(const at::Tensor& a, const at::Tensor& b) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda(), "gemm operands must be CUDA tensors");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm expects bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "gemm shape mismatch");
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous(), "gemm operands must be contiguous");
  TORCH_CHECK(a.size(1) % 8 == 0, "K must be a multiple of 8 (16-byte TMA row stride)");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0,
              "gemm operands must be 16-byte aligned");
}

// Shared launch path of the plain and SiLU-mul GEMMs.
static void run_gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int epilogue, int force_splits,
                     unsigned long long* dbg) {
  const int M = a.size(0), N = b.size(0);
  const int out_cols = out.size(1);
  Plan p = plan_gemm(a, b, false, force_splits, /*halve_tokens=*/force_splits == 0);
  const int kb_total = (int(a.size(1)) + BK - 1) / BK;
  // two CTAs per weight tile (split K over a cluster pair) when the doubled grid still fits in a
  // wave and the token tile is narrow (measured: a win up to 32 tokens, a loss at 128, where
  // exchanging the 64 KB partial tile costs more than halving each CTA's weight stream saves)
  const bool pair = p.swap && force_splits == 0 && gemm_pair_enabled() && kb_total >= 4 && p.bn <= 32 &&
                    p.tiles_p * p.tiles_q * 2 <= num_sms();
  if (pair) {
    p.kb_per = (kb_total + 1) / 2;
    p.splits = 2;
  }
  GemmArgs args = {};
  args.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  args.K = a.size(1);
  args.ldo = out_cols;
  args.kb_per_split = p.kb_per;
  args.dbg = dbg;
  if (p.swap) { args.P_rows = N; args.Q_rows = M; } else { args.P_rows = M; args.Q_rows = N; }
  at::Tensor ws;
  if (p.splits > 1 && !pair) {
    ws = at::empty({int64_t(p.tiles_p) * p.tiles_q * p.splits * BM * p.bn}, a.options().dtype(at::kFloat));
    args.ws = ws.data_ptr<float>();
    args.counters = counter_slot();
  }
  CUtensorMap to = p.tp;
  if (p.swap) {
    TORCH_CHECK(out_cols % 8 == 0, "swap-AB GEMM output width must be a multiple of 8 (16-byte rows)");
    to = make_store_map(out.data_ptr(), M, out_cols, epilogue == kSiluMul ? 64 : BM, pair ? p.bn / 2 : p.bn);
  } else if (out_map_ok(out.data_ptr(), out_cols, false)) {
    to = make_out_map_sw128(out.data_ptr(), M, out_cols, false);
    args.tma_out = true;
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (pair) {
    if (epilogue == kSiluMul) TORCH_CHECK(N % 128 == 0, "packed gate/up rows must be a multiple of 128");
#define ISB_PAIR(BN_)                                                                                   \
  if (p.bn == BN_) {                                                                                    \
    if (epilogue == kStore) launch_gemm_pair<BN_, kStore>(p.tp, p.tq, to, args, p.tiles_p, p.tiles_q, st); \
    else launch_gemm_pair<BN_, kSiluMul>(p.tp, p.tq, to, args, p.tiles_p, p.tiles_q, st);                   \
    return;                                                                                             \
  }
    ISB_PAIR(16) ISB_PAIR(32) ISB_PAIR(64) ISB_PAIR(128)
#undef ISB_PAIR
    TORCH_CHECK(false, "unsupported tile width");
  }
  if (epilogue == kStore) {
    if (p.swap) dispatch_bn<kStore, true>(p.bn, p.tp, p.tq, to, args, p.tiles_p, p.tiles_q, p.splits, st);
    else launch_gemm<256, false, kStore>(p.tp, p.tq, to, args, p.tiles_p, p.tiles_q, p.splits, st);
  } else {
    TORCH_CHECK(N % 128 == 0 || !p.swap, "packed gate/up rows must be a multiple of 128");
    if (p.swap) dispatch_bn<kSiluMul, true>(p.bn, p.tp, p.tq, to, args, p.tiles_p, p.tiles_q, p.splits, st);
    else launch_gemm<256, false, kSiluMul>(p.tp, p.tq, to, args, p.tiles_p, p.tiles_q, p.splits, st);
  }
}

// acc[M, N] (fp32) += a[M, K] . b[N, K]^T.  Every CTA (including every split-K
// slice) adds its tile with vector atomics, so the split count only sets the
// parallelism; the consumer of ``acc`` is expected to read and re-zero it.
void gemm_accum(const at::Tensor& a_in, const at::Tensor& b, at::Tensor acc, int64_t splits) {
  at::Tensor a = a_in.contiguous();
  check_operands(a, b);
  const int M = a.size(0), N = b.size(0);
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.size(0) >= M && acc.size(1) == N,
              "accumulator must be contiguous fp32 [>= M, N]");
  if (M == 0) return;
  const int kb_total = (int(a.size(1)) + BK - 1) / BK;
  Plan p = plan_gemm(a, b, false, 1);
  int sp = splits > 0 ? int(splits) : 1;
  if (splits <= 0) {  // fill the machine: one to two waves of CTAs
    const int tiles = p.tiles_p * p.tiles_q;
    while (sp < 16 && tiles * sp * 2 <= 2 * num_sms() && kb_total / (sp * 2) >= 2) sp *= 2;
  }
  p.kb_per = (kb_total + sp - 1) / sp;
  p.splits = (kb_total + p.kb_per - 1) / p.kb_per;
  GemmArgs args = {};
  args.acc = acc.data_ptr<float>();
  args.K = a.size(1);
  args.ldo = N;
  args.kb_per_split = p.kb_per;
  args.acc_plain = p.splits == 1;
  if (p.swap) { args.P_rows = N; args.Q_rows = M; } else { args.P_rows = M; args.Q_rows = N; }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (p.swap) {
    // the bulk reduce-add needs 16-byte rows; other widths add from registers
    const bool bulk = N % 4 == 0 && (reinterpret_cast<uintptr_t>(acc.data_ptr()) & 15) == 0;
    if (!bulk) args.acc_direct = true;
    const CUtensorMap tacc = bulk ? make_acc_map(acc.data_ptr(), M, N, BM, p.bn) : p.tp;
    dispatch_bn<kRedAdd, true>(p.bn, p.tp, p.tq, tacc, args, p.tiles_p, p.tiles_q, p.splits, st);
  }
  else {
    const bool bulk = out_map_ok(acc.data_ptr(), N, true);
    args.tma_out = bulk;
    const CUtensorMap tacc = bulk ? make_out_map_sw128(acc.data_ptr(), M, N, true) : p.tp;
    launch_gemm<256, false, kRedAdd>(p.tp, p.tq, tacc, args, p.tiles_p, p.tiles_q, p.splits, st);
  }
}

at::Tensor add_rmsnorm_acc(at::Tensor acc, at::Tensor residual, const at::Tensor& w, double eps, bool zc);

// ``out = RMSNorm(residual + a . b^T)`` with ``residual`` updated and ``acc`` (fp32 [>= M, N], zero
// between uses) re-zeroed, in ONE kernel when the split-K grid fits on the SMs at once (the add and
// the norm run after an in-kernel grid barrier); otherwise the accumulate GEMM and the separate
// add + RMSNorm kernel.
at::Tensor gemm_accum_norm(const at::Tensor& a_in, const at::Tensor& b, at::Tensor acc, at::Tensor residual,
                           const at::Tensor& w, double eps, bool zc) {
  at::Tensor a = a_in.contiguous();
  check_operands(a, b);
  const int M = a.size(0), N = b.size(0);
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.size(0) >= M && acc.size(1) == N,
              "accumulator must be contiguous fp32 [>= M, N]");
  TORCH_CHECK(residual.scalar_type() == at::kBFloat16 && residual.is_contiguous() && residual.size(0) == M &&
                  residual.size(1) == N && N % 8 == 0, "residual must be contiguous bf16 [M, N], N % 8 == 0");
  at::Tensor out = at::empty_like(residual);
  if (M == 0) return out;
  const int kb_total = (int(a.size(1)) + BK - 1) / BK;
  Plan p = plan_gemm(a, b, false, 1);
  const int tiles = p.tiles_p * p.tiles_q;
  static const bool enabled = [] {
    const char* e = std::getenv("ISB_FUSED_NORM");
    return !(e && e[0] == '0');
  }();
  if (!enabled || tiles > num_sms()) {  // the grid barrier needs every CTA resident
    gemm_accum(a, b, acc, 0);
    return add_rmsnorm_acc(acc, residual, w, eps, zc);
  }
  // one wave: as many K splits as fit next to the tiles (each split keeps >= 2 k-blocks)
  const int sp = std::max(1, std::min({16, num_sms() / tiles, kb_total / 2}));
  p.kb_per = (kb_total + sp - 1) / sp;
  p.splits = (kb_total + p.kb_per - 1) / p.kb_per;
  GemmArgs args = {};
  args.acc = acc.data_ptr<float>();
  args.K = a.size(1);
  args.ldo = N;
  args.kb_per_split = p.kb_per;
  args.acc_plain = p.splits == 1;
  args.counters = counter_slot();
  args.norm_out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  args.norm_res = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  args.norm_w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  args.norm_eps = float(eps);
  args.norm_zc = zc;
  args.norm_rows = M;
  if (p.swap) { args.P_rows = N; args.Q_rows = M; } else { args.P_rows = M; args.Q_rows = N; }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (p.swap) {
    // the bulk reduce-add needs 16-byte rows; other widths add from registers
    const bool bulk = N % 4 == 0 && (reinterpret_cast<uintptr_t>(acc.data_ptr()) & 15) == 0;
    if (!bulk) args.acc_direct = true;
    const CUtensorMap tacc = bulk ? make_acc_map(acc.data_ptr(), M, N, BM, p.bn) : p.tp;
    dispatch_bn<kRedAdd, true>(p.bn, p.tp, p.tq, tacc, args, p.tiles_p, p.tiles_q, p.splits, st);
  }
  else {
    const bool bulk = out_map_ok(acc.data_ptr(), N, true);
    args.tma_out = bulk;
    const CUtensorMap tacc = bulk ? make_out_map_sw128(acc.data_ptr(), M, N, true) : p.tp;
    launch_gemm<256, false, kRedAdd>(p.tp, p.tq, tacc, args, p.tiles_p, p.tiles_q, p.splits, st);
  }
  return out;
}

// Tensor-parallel row-parallel GEMM fused with the reduce-scatter (or, ``one_shot``, with the
// all-to-all push of a one-shot all-reduce: every row to every rank).  ``a`` [T, K/W] . ``b`` [H, K/W]^T
// is this rank's partial product.  Token rows [r*own_rows, (r+1)*own_rows) belong to rank r: each
// complete bf16 row goes straight into rank r's slot for this rank (``slots``: int64 [W] device
// table of the ranks' slot arrays [W][slot_rows][H] bf16, peer memory included), so a partial
// crosses NVLink once, as bf16, with plain stores.  Split-K CTAs first reduce into ``staging``
// (this rank's fp32 [>= T, H], zero between uses; the tile's last CTA re-zeroes it).  The grid's
// last CTA then bumps every rank's arrival counter (``flags``: int64 [W] device addresses), which
// the owner's ``tp_norm_allgather`` waits for.
int64_t tp_gemm_rs(const at::Tensor& a_in, const at::Tensor& b, const at::Tensor& slots, int64_t slot_rows,
                   at::Tensor staging, const at::Tensor& flags, int64_t rank, int64_t own_rows, int64_t splits,
                   bool one_shot) {
  at::Tensor a = a_in.contiguous();
  check_operands(a, b);
  const int M = a.size(0), N = b.size(0);
  TORCH_CHECK(slots.scalar_type() == at::kLong && flags.scalar_type() == at::kLong && slots.numel() == flags.numel() &&
                  slots.is_cuda() && flags.is_cuda(), "slots / flags: int64 device tables, one entry per rank");
  TORCH_CHECK(staging.scalar_type() == at::kFloat && staging.is_contiguous() && staging.size(0) >= M &&
                  staging.size(1) == N, "staging accumulator must be contiguous fp32 [>= T, H]");
  TORCH_CHECK(rank >= 0 && rank < slots.numel(), "rank out of range");
  TORCH_CHECK(one_shot ? M <= slot_rows
                       : own_rows > 0 && own_rows <= slot_rows && int64_t(own_rows) * slots.numel() >= M,
              "every token row needs an owner rank and a slot row");
  TORCH_CHECK(N % 128 == 0, "output features must be a multiple of 128 (whole 128-feature tiles)");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(staging.data_ptr()) & 15) == 0, "staging rows must be 16-byte aligned");
  if (M == 0) return 0;
  const int kb_total = (int(a.size(1)) + BK - 1) / BK;
  Plan p = plan_gemm(a, b, false, 1);
  // swap-AB tiles reduce their K splits inside one cluster (at most 8 CTAs, one wave of SMs)
  static const bool rs_cluster = [] {
    const char* e = std::getenv("ISB_RS_CLUSTER");
    return !(e && e[0] == '0');
  }();
  const bool clustered = p.swap && rs_cluster;
  int sp = splits > 0 ? int(splits) : 1;
  if (splits <= 0) {
    const int tiles = p.tiles_p * p.tiles_q;
    if (clustered) {
      sp = std::max(1, std::min({8, num_sms() / std::max(tiles, 1), kb_total}));
    } else {
      while (sp < 16 && tiles * sp * 2 <= 2 * num_sms() && kb_total / (sp * 2) >= 2) sp *= 2;
    }
  }
  if (clustered) sp = std::min(sp, 8);
  p.kb_per = (kb_total + sp - 1) / sp;
  p.splits = (kb_total + p.kb_per - 1) / p.kb_per;
  TORCH_CHECK(p.tiles_p * p.tiles_q <= kCountersPerSlot || p.splits == 1, "too many split-K tiles");
  GemmArgs args = {};
  args.K = a.size(1);
  args.ldo = N;
  args.kb_per_split = p.kb_per;
  args.acc = staging.data_ptr<float>();
  args.counters = p.splits > 1 ? counter_slot() : nullptr;
  args.dsts = reinterpret_cast<const unsigned long long*>(slots.data_ptr<int64_t>());
  args.ndst = int(slots.numel());
  args.own_rows = one_shot ? M : int(own_rows);
  args.slot_rows = int(slot_rows);
  args.bcast = one_shot;
  args.peer_flags = reinterpret_cast<const unsigned long long*>(flags.data_ptr<int64_t>());
  args.rank = int(rank);
  if (p.swap) { args.P_rows = N; args.Q_rows = M; } else { args.P_rows = M; args.Q_rows = N; }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (clustered && p.splits > 1) {
    switch (p.bn) {
      case 16: launch_rs_cluster<16>(p.tp, p.tq, args, p.tiles_p, p.tiles_q, p.splits, st); break;
      case 32: launch_rs_cluster<32>(p.tp, p.tq, args, p.tiles_p, p.tiles_q, p.splits, st); break;
      case 64: launch_rs_cluster<64>(p.tp, p.tq, args, p.tiles_p, p.tiles_q, p.splits, st); break;
      case 128: launch_rs_cluster<128>(p.tp, p.tq, args, p.tiles_p, p.tiles_q, p.splits, st); break;
      default: TORCH_CHECK(false, "unsupported tile width");
    }
  } else if (p.swap) {  // split-K partials of a swap-AB tile meet in the staging rows by bulk reduce-add
    const CUtensorMap tst = p.splits > 1 ? make_acc_map(staging.data_ptr(), M, N, BM, p.bn) : p.tp;
    dispatch_bn<kRsPush, true>(p.bn, p.tp, p.tq, tst, args, p.tiles_p, p.tiles_q, p.splits, st);
  } else {
    launch_gemm<256, false, kRsPush>(p.tp, p.tq, p.tp, args, p.tiles_p, p.tiles_q, p.splits, st);
  }
  return int64_t(p.tiles_p) * p.tiles_q * p.splits;  // CTAs: each bumps every rank's counter once
}

int64_t comm_error_word_address();

// One-shot exchange in ONE kernel (decode, swap-AB tiles, at most 128 tokens): the row-parallel
// GEMM reduces its K splits in a cluster, pushes every row to every rank's slot, waits (bounded)
// until all ranks' CTAs have pushed, then adds the residual and applies the RMSNorm of all rows
// into ``xout`` (and ``residual``).  Every CTA of the grid must be resident at once: the split
// count keeps the grid within one wave of SMs.
void tp_gemm_rs_norm(const at::Tensor& a_in, const at::Tensor& b, const at::Tensor& slots, int64_t slot_rows,
                     const at::Tensor& flags, int64_t rank, const at::Tensor& slots_local, at::Tensor residual,
                     const at::Tensor& w, at::Tensor xout, at::Tensor ctl, double eps, bool zc) {
  at::Tensor a = a_in.contiguous();
  check_operands(a, b);
  const int M = a.size(0), N = b.size(0);
  TORCH_CHECK(M <= 128 && M <= slot_rows, "fused one-shot exchange serves at most 128 tokens");
  TORCH_CHECK(N % 128 == 0 && N <= 1024, "fused one-shot exchange: hidden size a multiple of 128, at most 1024");
  TORCH_CHECK(slots.scalar_type() == at::kLong && flags.scalar_type() == at::kLong && slots.numel() == flags.numel() &&
                  slots.numel() <= 8, "slots / flags: int64 device tables, one entry per rank (<= 8)");
  TORCH_CHECK(residual.scalar_type() == at::kBFloat16 && residual.is_contiguous() && residual.size(0) >= M &&
                  residual.size(1) == N, "residual must be contiguous bf16 [>= T, H]");
  TORCH_CHECK(xout.scalar_type() == at::kBFloat16 && xout.is_contiguous() && xout.size(0) >= M && xout.size(1) == N,
              "output must be contiguous bf16 [>= T, H]");
  TORCH_CHECK(ctl.scalar_type() == at::kInt && ctl.numel() >= 8, "control words: int32 [8]");
  if (M == 0) return;
  const int kb_total = (int(a.size(1)) + BK - 1) / BK;
  Plan p = plan_gemm(a, b, false, 1);
  TORCH_CHECK(p.swap, "fused one-shot exchange needs swap-AB tiles");
  const int tiles = p.tiles_p * p.tiles_q;
  const int sp = std::max(1, std::min({8, num_sms() / std::max(tiles, 1), kb_total}));
  p.kb_per = (kb_total + sp - 1) / sp;
  p.splits = (kb_total + p.kb_per - 1) / p.kb_per;
  TORCH_CHECK(tiles * p.splits <= num_sms(), "fused exchange grid must fit on the SMs");
  GemmArgs args = {};
  args.K = a.size(1);
  args.ldo = N;
  args.kb_per_split = p.kb_per;
  args.dsts = reinterpret_cast<const unsigned long long*>(slots.data_ptr<int64_t>());
  args.ndst = int(slots.numel());
  args.own_rows = M;
  args.slot_rows = int(slot_rows);
  args.bcast = true;
  args.peer_flags = reinterpret_cast<const unsigned long long*>(flags.data_ptr<int64_t>());
  args.rank = int(rank);
  args.tp_slots = reinterpret_cast<const __nv_bfloat16*>(slots_local.data_ptr());
  args.tp_ctl = reinterpret_cast<unsigned int*>(ctl.data_ptr<int>());
  args.tp_err = reinterpret_cast<unsigned int*>(comm_error_word_address());
  args.norm_out = reinterpret_cast<__nv_bfloat16*>(xout.data_ptr());
  args.norm_res = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  args.norm_w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  args.norm_eps = float(eps);
  args.norm_zc = zc;
  args.norm_rows = M;
  args.P_rows = N;
  args.Q_rows = M;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (p.splits > 1) {
    switch (p.bn) {
      case 16: launch_rs_cluster<16>(p.tp, p.tq, args, p.tiles_p, p.tiles_q, p.splits, st); break;
      case 32: launch_rs_cluster<32>(p.tp, p.tq, args, p.tiles_p, p.tiles_q, p.splits, st); break;
      case 64: launch_rs_cluster<64>(p.tp, p.tq, args, p.tiles_p, p.tiles_q, p.splits, st); break;
      case 128: launch_rs_cluster<128>(p.tp, p.tq, args, p.tiles_p, p.tiles_q, p.splits, st); break;
      default: TORCH_CHECK(false, "unsupported tile width");
    }
  } else {
    dispatch_bn<kRsPush, true>(p.bn, p.tp, p.tq, p.tp, args, p.tiles_p, p.tiles_q, 1, st);
  }
}

at::Tensor gemm(const at::Tensor& a_in, const at::Tensor& b, int64_t epilogue, int64_t splits) {
  at::Tensor a = a_in.contiguous();
  check_operands(a, b);
  const int M = a.size(0), N = b.size(0);
  TORCH_CHECK(epilogue == kStore || epilogue == kSiluMul, "gemm: unknown epilogue");
  at::Tensor out = at::empty({M, epilogue == kSiluMul ? N / 2 : N}, a.options());
  if (M == 0) return out;
  run_gemm(a, b, out, int(epilogue), int(splits), nullptr);
  return out;
}

// Diagnostics: the accumulating GEMM (``acc`` fp32 [>= M, N], zero between uses) with per-CTA
// phase timestamps as ``gemm_timeline``.
at::Tensor gemm_accum_timeline(const at::Tensor& a_in, const at::Tensor& b, at::Tensor acc, int64_t splits) {
  at::Tensor a = a_in.contiguous();
  check_operands(a, b);
  const int M = a.size(0), N = b.size(0);
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.size(0) >= M && acc.size(1) == N,
              "accumulator must be contiguous fp32 [>= M, N]");
  const int kb_total = (int(a.size(1)) + BK - 1) / BK;
  Plan p = plan_gemm(a, b, false, 1);
  const int sp = std::max(1, int(splits <= -3000 ? -(splits + 3000) : splits <= -2000 ? -(splits + 2000)
                                 : splits <= -1000 ? -(splits + 1000) : splits < 0 ? -splits : splits));
  p.kb_per = (kb_total + sp - 1) / sp;
  p.splits = (kb_total + p.kb_per - 1) / p.kb_per;
  at::Tensor ts = at::zeros({int64_t(p.tiles_p) * p.tiles_q * p.splits, 8}, a.options().dtype(at::kLong));
  GemmArgs args = {};
  args.acc = acc.data_ptr<float>();
  args.K = a.size(1);
  args.ldo = N;
  args.kb_per_split = p.kb_per;
  args.acc_plain = p.splits == 1;
  args.acc_direct = splits < 0;
  if (splits <= -1000) {  // -1000 - s: TMEM loads only; -2000 - s: stores only; -3000 - s: 17 x stores
    args.epi_probe = splits <= -3000 ? 3 : splits <= -2000 ? 2 : 1;
  }
  args.dbg = reinterpret_cast<unsigned long long*>(ts.data_ptr());
  if (p.swap) { args.P_rows = N; args.Q_rows = M; } else { args.P_rows = M; args.Q_rows = N; }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (p.swap) {
    // the bulk reduce-add needs 16-byte rows; other widths add from registers
    const bool bulk = N % 4 == 0 && (reinterpret_cast<uintptr_t>(acc.data_ptr()) & 15) == 0;
    if (!bulk) args.acc_direct = true;
    const CUtensorMap tacc = bulk ? make_acc_map(acc.data_ptr(), M, N, BM, p.bn) : p.tp;
    dispatch_bn<kRedAdd, true>(p.bn, p.tp, p.tq, tacc, args, p.tiles_p, p.tiles_q, p.splits, st);
  }
  else {
    const bool bulk = out_map_ok(acc.data_ptr(), N, true);
    args.tma_out = bulk;
    const CUtensorMap tacc = bulk ? make_out_map_sw128(acc.data_ptr(), M, N, true) : p.tp;
    launch_gemm<256, false, kRedAdd>(p.tp, p.tq, tacc, args, p.tiles_p, p.tiles_q, p.splits, st);
  }
  return ts;
}

// Diagnostics: run the plain GEMM and return per-CTA phase timestamps (ns, %globaltimer):
// [entry, setup done, first TMA issued, first stage landed, last MMA issued, accumulator ready,
//  epilogue done, exit].
at::Tensor gemm_timeline(const at::Tensor& a_in, const at::Tensor& b, int64_t splits) {
  at::Tensor a = a_in.contiguous();
  check_operands(a, b);
  const int M = a.size(0), N = b.size(0);
  if (splits < 0) {  // LM-head argmax epilogue (greedy)
    Plan p = plan_gemm(a, b, false);
    at::Tensor ts = at::zeros({int64_t(p.tiles_p) * p.tiles_q, 8}, a.options().dtype(at::kLong));
    const int vtiles = p.swap ? p.tiles_p : p.tiles_q;
    at::Tensor pv = at::empty({vtiles, M}, a.options().dtype(at::kFloat));
    at::Tensor pi = at::empty({vtiles, M}, a.options().dtype(at::kInt));
    at::Tensor temps = at::zeros({M}, a.options().dtype(at::kFloat));
    at::Tensor rng = at::zeros({2}, a.options().dtype(at::kInt));
    GemmArgs args = {};
    args.K = a.size(1);
    args.kb_per_split = p.kb_per;
    args.temps = temps.data_ptr<float>();
    args.rng = rng.data_ptr<int>();
    args.part_val = pv.data_ptr<float>();
    args.part_idx = pi.data_ptr<int>();
    args.dbg = reinterpret_cast<unsigned long long*>(ts.data_ptr());
    cudaStream_t st = at::cuda::getCurrentCUDAStream();
    if (p.swap) {
      args.P_rows = N; args.Q_rows = M;
      dispatch_bn<kArgmax, true>(p.bn, p.tp, p.tq, p.tp, args, p.tiles_p, p.tiles_q, 1, st);
    } else {
      args.P_rows = M; args.Q_rows = N;
      launch_gemm<256, false, kArgmax>(p.tp, p.tq, p.tp, args, p.tiles_p, p.tiles_q, 1, st);
    }
    return ts;
  }
  at::Tensor out = at::empty({M, N}, a.options());
  // the same plan run_gemm makes (two token tiles per weight tile when it halves them, a cluster
  // pair for narrow tiles): one row of timestamps per CTA it may launch (unused rows stay zero)
  Plan p = plan_gemm(a, b, false, int(splits), /*halve_tokens=*/splits == 0);
  const int64_t ctas = int64_t(p.tiles_p) * p.tiles_q * std::max(p.splits, 2);
  at::Tensor ts = at::zeros({ctas, 8}, a.options().dtype(at::kLong));
  run_gemm(a, b, out, kStore, int(splits), reinterpret_cast<unsigned long long*>(ts.data_ptr()));
  return ts;
}

static bool lm_persistent_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("ISB_LM_PERSISTENT");
    return !(e && e[0] == '0');
  }();
  return on;
}

std::tuple<at::Tensor, at::Tensor> lm_head_sample(const at::Tensor& h_in, const at::Tensor& w, const at::Tensor& temps,
                                                  const at::Tensor& rng, int64_t vocab_offset) {
  at::Tensor h = h_in.contiguous();
  check_operands(h, w);
  TORCH_CHECK(temps.scalar_type() == at::kFloat && rng.scalar_type() == at::kInt, "temps fp32 / rng int32");
  const int B = h.size(0), V = w.size(0);
  at::Tensor val = at::empty({B}, h.options().dtype(at::kFloat));
  at::Tensor idx = at::empty({B}, h.options().dtype(at::kInt));
  if (B == 0) return {val, idx};
  Plan p = plan_gemm(h, w, false);
  const int vtiles = p.swap ? p.tiles_p : p.tiles_q;
  at::Tensor pv = at::empty({vtiles, B}, val.options());
  at::Tensor pi = at::empty({vtiles, B}, idx.options());
  GemmArgs args = {};
  args.K = h.size(1);
  args.kb_per_split = p.kb_per;
  args.temps = temps.data_ptr<float>();
  args.rng = rng.data_ptr<int>();
  args.part_val = pv.data_ptr<float>();
  args.part_idx = pi.data_ptr<int>();
  args.vocab_offset = int(vocab_offset);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (p.swap && p.tiles_q == 1 && lm_persistent_enabled()) {
    args.P_rows = V; args.Q_rows = B;
    switch (p.bn) {
      case 16: launch_lm_persistent<16>(p.tp, p.tq, args, p.tiles_p, st); break;
      case 32: launch_lm_persistent<32>(p.tp, p.tq, args, p.tiles_p, st); break;
      case 64: launch_lm_persistent<64>(p.tp, p.tq, args, p.tiles_p, st); break;
      default: launch_lm_persistent<128>(p.tp, p.tq, args, p.tiles_p, st); break;
    }
  } else if (p.swap) {
    args.P_rows = V; args.Q_rows = B;
    dispatch_bn<kArgmax, true>(p.bn, p.tp, p.tq, p.tp, args, p.tiles_p, p.tiles_q, 1, st);
  } else {
    args.P_rows = B; args.Q_rows = V;
    launch_gemm<256, false, kArgmax>(p.tp, p.tq, p.tp, args, p.tiles_p, p.tiles_q, 1, st);
  }
  launch_pdl(argmax_tiles_kernel, dim3(B), dim3(256), 0, st, pv.data_ptr<float>(), pi.data_ptr<int>(), vtiles, B, int(vocab_offset),
                                         val.data_ptr<float>(), idx.data_ptr<int>());
  return {val, idx};
}

int64_t gemm_error_word() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_err, sizeof(v));
  const unsigned int z = 0;
  cudaMemcpyToSymbol(g_gemm_err, &z, sizeof(z));
  return v;
}

// Device address of the error word (read by the per-step status kernel).
int64_t gemm_error_word_address() {
  void* p = nullptr;
  TORCH_CHECK(cudaGetSymbolAddress(&p, g_gemm_err) == cudaSuccess, "error word address");
  return reinterpret_cast<int64_t>(p);
}

}  // namespace isb
