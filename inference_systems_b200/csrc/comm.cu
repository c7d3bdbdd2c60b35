// Tensor-parallel communication over NVLink peer memory.
//
// Symmetric buffers: every rank cudaMalloc's one region, exports a CUDA IPC
// handle, and maps every peer's region (``symm_alloc`` / ``symm_open``); kernels
// then address peers with plain device pointers (P2P loads, stores and red
// atomics through NVSwitch).  Synchronisation between ranks uses monotone
// counters in the symmetric region that other ranks bump with system-scope
// releases; every wait polls THIS rank's memory (no NVLink round trip per poll)
// and is bounded by a %globaltimer deadline (``comm_set_wait_timeout``); a
// timeout records an error word (``comm_error_word``) and later waits return at
// once, so a missing peer can never hang a GPU.
//
//  * tp_norm_allgather: second half of the fused row-parallel exchange.  The
//    row-parallel GEMM (gemm.cu ``tp_gemm_rs``) reduce-scattered its partial
//    product by token: every rank stored the complete bf16 rows owned by rank r
//    into rank r's slot for that source, then bumped rank r's arrival counter.
//    This kernel waits until all W ranks have arrived, and for each owned row
//    sums the W slots in fp32, adds the residual, applies the next RMSNorm and
//    pushes the normalised bf16 row into every rank's activation buffer (the
//    all-gather, P2P stores), then releases every rank's gather counter; its
//    last CTA waits for all owners' pushes, so the next kernel (a column-parallel
//    GEMM, PDL-launched) reads a complete, local activation.  Per exchange a rank
//    sends (W-1)/W * T * H bf16 partial sums and (W-1) * T/W * H bf16 activations.
//  * xrank_argmax: cross-rank (score, token) argmax of the vocab-parallel LM
//    head; each rank publishes 8 bytes per row to every peer instead of gathering logits.

#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "launch.cuh"

namespace isb {

__device__ unsigned int g_comm_err;
// Deadline of every cross-rank wait in this file (ns).
__device__ unsigned long long g_comm_wait_ns = 2000000000ull;

namespace {

ISB_DEVICE unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

ISB_DEVICE bool comm_failed() { return *reinterpret_cast<volatile unsigned int*>(&g_comm_err) != 0u; }

// Wait until flags[0..n) are all >= 1 (bounded).  Returns false on timeout.
ISB_DEVICE bool wait_flags(const unsigned int* flags, int n) {
  if (comm_failed()) return false;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = *reinterpret_cast<volatile unsigned long long*>(&g_comm_wait_ns);
  for (int r = 0; r < n; ++r) {
    uint32_t spins = 0;
    while (ld_acquire_sys(flags + r) < 1u) {
      if ((++spins & 1023u) == 0 && globaltimer_ns() - t0 > limit) {
        atomicOr(&g_comm_err, 1u);
        return false;
      }
    }
  }
  return true;
}

// Wait until the local counter ``*cnt`` has reached ``target`` (wrap-safe, bounded).  ``code`` is
// OR'ed into the error word on timeout.
ISB_DEVICE bool wait_geq(const unsigned int* cnt, unsigned int target, unsigned int code) {
  if (comm_failed()) return false;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = *reinterpret_cast<volatile unsigned long long*>(&g_comm_wait_ns);
  uint32_t spins = 0;
  while (int(ld_acquire_sys(cnt) - target) < 0) {
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > limit) {
      atomicOr(&g_comm_err, code);
      return false;
    }
  }
  return true;
}

constexpr int kMaxWorld = 8;
constexpr int kMaxChunks = 4;  // columns per thread / 8: H <= 4 * 8 * 512

// Owned rows are spread over the grid (blockDim = H / 8 rounded up to a warp, at most 512; 8
// columns per thread per chunk).  ``slots``: this rank's [world][slot_rows][H] bf16 partial sums;
// row i of each source slot is token ``lo + i``.  ``ctl`` words: 0 arrivals of row-parallel GEMM
// CTAs, 1 arrivals of owner CTAs, 2 / 3 the targets those counters reached at the end of the
// previous exchange, 4 this kernel's CTA-completion counter.  ``rs_incr`` / ``ag_incr``: arrivals
// this exchange adds to words 0 / 1.
__global__ void __launch_bounds__(512) tp_norm_ag_kernel(
    const __nv_bfloat16* __restrict__ slots, int slot_rows, __nv_bfloat16* __restrict__ residual,
    const __nv_bfloat16* __restrict__ w, const unsigned long long* __restrict__ xdst,
    const unsigned long long* __restrict__ ag_flags, unsigned int* ctl, int lo, int rows, int H, float eps,
    bool zc, int world, bool wait_gather, unsigned int rs_incr, unsigned int ag_incr, int one_shot_rank) {
  pdl_trigger();
  pdl_wait();
  __shared__ int s_ok;
  __shared__ float red[16];
  __shared__ unsigned long long s_x[kMaxWorld];  // activation buffers, read once
  const int tid = threadIdx.x, nt = blockDim.x;
  if (tid < world) s_x[tid] = xdst[tid];
  // targets of this exchange; the previous exchange's last CTA wrote the bases before its grid
  // completed (ordered by pdl_wait), and this exchange's last CTA moves them only after every CTA
  // has read them
  const unsigned int rs_target = ctl[2] + rs_incr, ag_target = ctl[3] + ag_incr;
  if (tid == 0) s_ok = rows > 0 ? (wait_geq(ctl, rs_target, 2u) ? 1 : 0) : 1;
  __syncthreads();
  const size_t slot_stride = size_t(slot_rows) * H;
  for (int i = blockIdx.x; i < rows; i += gridDim.x) {
    const size_t r = size_t(lo) + i;
    __nv_bfloat16* res = residual + r * H;
    const __nv_bfloat16* mine = slots + size_t(i) * H;
    float v[kMaxChunks][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = (tid + k * nt) * 8;
      if (c >= H) break;
      // every source's slice first (written by other GPUs: read from L2, never a stale L1 line),
      // so a thread has all of them in flight before it sums
      uint4 raw[kMaxWorld];
#pragma unroll
      for (int q = 0; q < kMaxWorld; ++q)
        raw[q] = q < world && s_ok ? __ldcg(reinterpret_cast<const uint4*>(mine + q * slot_stride + c))
                                   : make_uint4(0u, 0u, 0u, 0u);
      const Vec8 rr = load8(res + c);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[k][e] = rr.v[e];
#pragma unroll
      for (int q = 0; q < kMaxWorld; ++q) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[q]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          v[k][2 * e] += f.x;
          v[k][2 * e + 1] += f.y;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int q = 0; q < (nt + 31) / 32; ++q) tot += red[q];
    __syncthreads();  // ``red`` is reused by the next row
    const float rs = rsqrtf(tot / float(H) + eps);
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = (tid + k * nt) * 8;
      if (c >= H) break;
      store8(res + c, v[k]);
      float y[8];
      norm8(y, v[k], w + c, rs, zc);
      uint4 out;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(y[2 * e], y[2 * e + 1]);
      if (one_shot_rank >= 0) {  // one-shot: every rank normalises every row itself
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(s_x[one_shot_rank]) + r * H + c) = out;
        continue;
      }
      // the all-gather: the row goes to every rank's activation buffer (staggered start)
      for (int q = 0; q < world; ++q) {
        const int dst = (i + q) % world;
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(s_x[dst]) + r * H + c) = out;
      }
    }
  }
  // Count this CTA in on every rank (a system-scope fence after the CTA barrier orders all its
  // threads' pushes); the last CTA here then moves the targets on and, unless told otherwise,
  // waits until every owner's rows have arrived, so the grid completes with the full activation.
  __syncthreads();
  if (tid == 0) {
    if (one_shot_rank < 0) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");  // one fence orders the pushes before every count
      for (int q = 0; q < world; ++q) {
        unsigned int* f = reinterpret_cast<unsigned int*>(ag_flags[q]);
        asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(f) : "memory");
      }
    }
    unsigned int prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ctl + 4) : "memory");
    if (prev == gridDim.x - 1) {
      ctl[4] = 0u;
      if (wait_gather && one_shot_rank < 0) wait_geq(ctl + 1, ag_target, 4u);
      ctl[2] = rs_target;
      ctl[3] = ag_target;
    }
  }
}

// Single CTA.  Publish this rank's (score, token) per row to every peer's exchange slot,
// signal, wait for all ranks, reduce (ties -> smaller token id), write token ids.
__global__ void xrank_argmax_kernel(const float* __restrict__ val, const int* __restrict__ idx, int B,
                                    const unsigned long long* xbufs, const unsigned long long* peer_flags,
                                    unsigned int* my_xbuf_flags, const float2* my_xbuf, int rank, int world,
                                    int max_rows, int* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  __shared__ int ok;
  for (int t = threadIdx.x; t < B; t += blockDim.x) {
    const float2 e = make_float2(val[t], __int_as_float(idx[t]));
    for (int r = 0; r < world; ++r)
      reinterpret_cast<float2*>(xbufs[r])[size_t(rank) * max_rows + t] = e;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < world; ++r) {
      unsigned int* flag = reinterpret_cast<unsigned int*>(peer_flags[r]) + rank;
      asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(flag) : "memory");
    }
    ok = wait_flags(my_xbuf_flags, world);
  }
  __syncthreads();
  for (int t = threadIdx.x; t < B; t += blockDim.x) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < world; ++r) {
      const float2 e = __ldcg(my_xbuf + size_t(r) * max_rows + t);
      const int i = __float_as_int(e.y);
      if (e.x > best || (e.x == best && i < bi)) { best = e.x; bi = i; }
    }
    out[t] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0 && ok)
    for (int r = 0; r < world; ++r) atomicSub(my_xbuf_flags + r, 1u);
}

// The step's output row for the host: out[0..n) = the sampled tokens, out[n] = bit i set when
// error word i (words[i], device addresses) is nonzero.  One launch and the token copy that
// already happens carry every kernel's error state back each step.
__global__ void step_status_kernel(const int* __restrict__ toks, int n, const unsigned long long* __restrict__ words,
                                   int nwords, int* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = toks[i];
  if (threadIdx.x == 0) {
    int bits = 0;
    for (int i = 0; i < nwords; ++i)
      if (*reinterpret_cast<volatile const unsigned int*>(words[i]) != 0u) bits |= 1 << i;
    out[n] = bits;
  }
}

}  // namespace

// ------------------------------------------------------------- host side
// Allocate a zeroed device region and return (uint8 tensor view, IPC handle bytes).
std::tuple<at::Tensor, at::Tensor> symm_alloc(int64_t nbytes) {
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, nbytes) == cudaSuccess, "symm_alloc: cudaMalloc failed");
  TORCH_CHECK(cudaMemset(p, 0, nbytes) == cudaSuccess, "symm_alloc: memset failed");
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, p) == cudaSuccess, "symm_alloc: cudaIpcGetMemHandle failed");
  int dev;
  cudaGetDevice(&dev);
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, dev);
  at::Tensor view = at::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
  at::Tensor handle = at::empty({int64_t(sizeof(h))}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(handle.data_ptr(), &h, sizeof(h));
  return {view, handle};
}

int64_t symm_open(const at::Tensor& handle) {
  TORCH_CHECK(handle.numel() == int64_t(sizeof(cudaIpcMemHandle_t)), "bad IPC handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  TORCH_CHECK(e == cudaSuccess, "symm_open: cudaIpcOpenMemHandle failed: ", cudaGetErrorString(e));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

// Owner side of the row-parallel exchange (see the file comment) for a ``T``-token exchange with
// ``own_rows`` token rows per rank (rank r owns [r*own_rows, (r+1)*own_rows) clipped to T).
// ``slots``: this rank's [W, slot_rows, H] bf16 partial sums; ``residual`` [T, H] bf16 (the owned
// rows are read and updated); ``xdst`` / ``ag_flags``: int64 [W] device tables of every rank's
// activation buffer [>= T, H] bf16 and owner-arrival counter; ``ctl``: this rank's int32 control
// words (see the kernel); ``rs_incr``: row-parallel GEMM arrivals per exchange (W x its CTAs).
// ``wait_gather`` false skips the final wait (single-GPU tests that emulate several ranks).
constexpr int kNormMaxCtas = 296;  // two per SM: one exchange's rows never need more

static int norm_ctas(int64_t rows) { return int(std::max<int64_t>(std::min<int64_t>(rows, kNormMaxCtas), 1)); }

void tp_norm_allgather(const at::Tensor& slots, at::Tensor residual, const at::Tensor& w, const at::Tensor& xdst,
                       const at::Tensor& ag_flags, at::Tensor ctl, int64_t T, int64_t own_rows, int64_t rank,
                       int64_t rs_incr, double eps, bool zc, bool wait_gather, bool one_shot) {
  TORCH_CHECK(residual.is_contiguous() && residual.scalar_type() == at::kBFloat16 && residual.dim() == 2 &&
                  residual.size(0) >= T, "residual must be contiguous bf16 [>= T, H]");
  const int H = residual.size(1);
  const int W = xdst.numel();
  TORCH_CHECK(xdst.scalar_type() == at::kLong && ag_flags.scalar_type() == at::kLong && ag_flags.numel() == W &&
                  W >= 1 && W <= kMaxWorld, "one activation buffer and counter per rank (<= 8)");
  TORCH_CHECK(rank >= 0 && rank < W && (one_shot || (own_rows >= 1 && own_rows * W >= T)),
              "every token row needs an owner");
  TORCH_CHECK(slots.scalar_type() == at::kBFloat16 && slots.is_contiguous() && slots.dim() == 3 &&
                  slots.size(0) == W && slots.size(2) == H && slots.size(1) >= (one_shot ? T : own_rows),
              "slots: contiguous bf16 [W, >= rows, H]");
  TORCH_CHECK(H % 8 == 0 && H <= 16384, "hidden size must be a multiple of 8 and at most 16384");
  TORCH_CHECK(ctl.scalar_type() == at::kInt && ctl.numel() >= 5 && ctl.is_contiguous(), "int32 control words");
  auto owned = [&](int64_t r) { return std::max<int64_t>(0, std::min<int64_t>(own_rows, T - r * own_rows)); };
  int64_t ag_incr = 0;  // every CTA of every rank's owner kernel signals every rank once (two-shot)
  if (!one_shot)
    for (int64_t r = 0; r < W; ++r) ag_incr += norm_ctas(owned(r));
  const int64_t rows = one_shot ? T : owned(rank);
  const int64_t lo = one_shot ? 0 : std::min<int64_t>(rank * own_rows, T);
  const int threads = std::min(512, ((H / 8 + 31) / 32) * 32);
  launch_pdl(tp_norm_ag_kernel, dim3(norm_ctas(rows)), dim3(threads), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(slots.data_ptr()), int(slots.size(1)),
             reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
             reinterpret_cast<const unsigned long long*>(xdst.data_ptr<int64_t>()),
             reinterpret_cast<const unsigned long long*>(ag_flags.data_ptr<int64_t>()),
             reinterpret_cast<unsigned int*>(ctl.data_ptr<int>()), int(lo), int(rows), H, float(eps), zc, W,
             wait_gather, static_cast<unsigned int>(rs_incr), static_cast<unsigned int>(ag_incr),
             one_shot ? int(rank) : -1);
}

at::Tensor xrank_argmax(const at::Tensor& val, const at::Tensor& idx, const at::Tensor& xbufs,
                        const at::Tensor& peer_flags, at::Tensor my_flags, const at::Tensor& my_xbuf, int64_t rank,
                        int64_t max_rows) {
  const int B = val.numel();
  TORCH_CHECK(B <= max_rows, "xrank_argmax: more rows than the exchange buffer holds");
  at::Tensor out = at::empty({B}, idx.options());
  launch_pdl(xrank_argmax_kernel, dim3(1), dim3(512), 0, at::cuda::getCurrentCUDAStream(), 
      val.data_ptr<float>(), idx.data_ptr<int>(), B, reinterpret_cast<const unsigned long long*>(xbufs.data_ptr<int64_t>()),
      reinterpret_cast<const unsigned long long*>(peer_flags.data_ptr<int64_t>()),
      reinterpret_cast<unsigned int*>(my_flags.data_ptr<int>()), reinterpret_cast<const float2*>(my_xbuf.data_ptr()),
      int(rank), int(xbufs.numel()), int(max_rows), out.data_ptr<int>());
  return out;
}

at::Tensor step_status(const at::Tensor& toks, const at::Tensor& words) {
  TORCH_CHECK(toks.scalar_type() == at::kInt && toks.is_contiguous() && toks.dim() == 1, "tokens: int32 [n]");
  TORCH_CHECK(words.scalar_type() == at::kLong && words.is_cuda() && words.numel() <= 31, "error word addresses");
  const int n = toks.numel();
  at::Tensor out = at::empty({n + 1}, toks.options());
  launch_pdl(step_status_kernel, dim3(1), dim3(256), 0, at::cuda::getCurrentCUDAStream(), toks.data_ptr<int>(), n,
             reinterpret_cast<const unsigned long long*>(words.data_ptr<int64_t>()), int(words.numel()),
             out.data_ptr<int>());
  return out;
}

int64_t comm_error_word() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_comm_err, sizeof(v));
  const unsigned int z = 0;
  cudaMemcpyToSymbol(g_comm_err, &z, sizeof(z));
  return v;
}

// Deadline of the cross-rank waits (ns) on the current device.  Tests shorten it to make a wait
// on a counter that never advances run out quickly.
void comm_set_wait_timeout(int64_t ns) {
  const unsigned long long v = static_cast<unsigned long long>(ns);
  TORCH_CHECK(ns > 0, "wait timeout must be positive");
  TORCH_CHECK(cudaMemcpyToSymbol(g_comm_wait_ns, &v, sizeof(v)) == cudaSuccess, "setting the wait timeout");
}

// Device address of the error word (for the per-step error status kernel).
int64_t comm_error_word_address() {
  void* p = nullptr;
  TORCH_CHECK(cudaGetSymbolAddress(&p, g_comm_err) == cudaSuccess, "comm error word address");
  return reinterpret_cast<int64_t>(p);
}

}  // namespace isb
