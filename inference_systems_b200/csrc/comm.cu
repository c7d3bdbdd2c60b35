// Tensor-parallel communication over NVLink peer memory.
//
// Symmetric buffers: every rank cudaMalloc's one region, exports a CUDA IPC
// handle, and maps every peer's region (``symm_alloc`` / ``symm_open``); kernels
// then address peers with plain device pointers (P2P loads and stores through
// NVSwitch).  Synchronisation between ranks uses monotone counters in the
// symmetric region, released at system scope by their owner and acquired by
// peers.  Every wait is bounded by a %globaltimer deadline; a timeout records an
// error word (read by ``comm_error_word``) and later waits return at once, so a
// missing peer can never hang a GPU.
//
//  * add_rmsnorm_acc_tp: second half of the fused row-parallel GEMM all-reduce.
//    Each rank's GEMM (gemm.cu ``tp_gemm_accum``) reduced its partial product
//    into its own fp32 accumulator and bumped its own counter; this kernel waits
//    until every peer's counter has reached this rank's, sums all ranks'
//    accumulators with P2P loads, adds the residual and applies the next
//    RMSNorm.  Accumulators alternate between two parities per call, and the
//    buffer of the previous call is re-zeroed here: every peer finished reading
//    it, because each peer's current GEMM started after its previous consumer.
//  * xrank_argmax: cross-rank (score, token) argmax of the vocab-parallel LM
//    head; each rank publishes 8 bytes per row to every peer instead of gathering logits.

#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "launch.cuh"

namespace isb {

__device__ unsigned int g_comm_err;

namespace {

ISB_DEVICE unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until flags[0..n) are all >= 1 (bounded).  Returns false on timeout.
ISB_DEVICE bool wait_flags(const unsigned int* flags, int n) {
  if (*reinterpret_cast<volatile unsigned int*>(&g_comm_err) != 0u) return false;
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < n; ++r) {
    uint32_t spins = 0;
    while (ld_acquire_sys(flags + r) < 1u) {
      if ((++spins & 1023u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicOr(&g_comm_err, 1u);
        return false;
      }
    }
  }
  return true;
}

struct Vec8 {
  float v[8];
};

__device__ __forceinline__ Vec8 load8(const __nv_bfloat16* p) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  Vec8 r;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    r.v[2 * i] = f.x;
    r.v[2 * i + 1] = f.y;
  }
  return r;
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = raw;
}

// Wait until every counter flags[r] (peer memory) has reached ``target`` (bounded).
ISB_DEVICE bool wait_counters(const unsigned long long* flags, int n, unsigned int target) {
  if (*reinterpret_cast<volatile unsigned int*>(&g_comm_err) != 0u) return false;
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < n; ++r) {
    const unsigned int* f = reinterpret_cast<const unsigned int*>(flags[r]);
    uint32_t spins = 0;
    while (int(ld_acquire_sys(f) - target) < 0) {
      if ((++spins & 1023u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicOr(&g_comm_err, 1u);
        return false;
      }
    }
  }
  return true;
}

// One block per row, 8 columns per thread (blockDim = H / 8 rounded up to a warp, at most
// 512).  Every peer's slice of a chunk is loaded before any of it is summed (the peer loop
// is unrolled over kMaxWorld with predication), so a thread has 2 x world NVLink loads in
// flight instead of one round trip per peer.
constexpr int kMaxWorld = 8;

// Wait (threads 0..world-1, one peer each) until every rank's counter flags[r] has reached
// this rank's own ``*my_flag``; returns the block-wide verdict.
__device__ __forceinline__ bool wait_all_ranks(const unsigned long long* flags, const unsigned int* my_flag,
                                               int world) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < world) {  // one NVLink round trip per peer, all in parallel
    const unsigned int target = ld_acquire_sys(my_flag);
    if (!wait_counters(flags + threadIdx.x, 1, target)) ok = 0;
  }
  __syncthreads();
  return ok != 0;
}

// out_row = RMSNorm(res_row + sum_r accs[r][acc_row]); res_row is updated in place.  With ``outs``
// (nout buffer bases, peer memory included) the row is written to row ``acc_row`` of every one of
// them instead of to ``out``.
__device__ __forceinline__ void pull_add_norm_row(const unsigned long long* __restrict__ accs, int world, bool ok,
                                                  size_t acc_row, __nv_bfloat16* __restrict__ res,
                                                  const __nv_bfloat16* __restrict__ w,
                                                  __nv_bfloat16* __restrict__ out, int H, float eps, bool zc,
                                                  const unsigned long long* outs = nullptr, int nout = 0) {
  __shared__ float red[32];
  const int tid = threadIdx.x, nt = blockDim.x;
  const float* peer[kMaxWorld];
#pragma unroll
  for (int r = 0; r < kMaxWorld; ++r) peer[r] = r < world ? reinterpret_cast<const float*>(accs[r]) + acc_row * H : nullptr;
  float ss = 0.f;
  constexpr int kMaxChunks = 4;  // H <= 4 * 8 * 512
  float v[kMaxChunks][8];
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = (tid + k * nt) * 8;
    if (c >= H) break;
    float4 lo[kMaxWorld], hi[kMaxWorld];
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r) {
      if (r < world && ok) {
        lo[r] = __ldcv(reinterpret_cast<const float4*>(peer[r] + c));
        hi[r] = __ldcv(reinterpret_cast<const float4*>(peer[r] + c + 4));
      } else {
        lo[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        hi[r] = lo[r];
      }
    }
    float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r) {
      x[0] += lo[r].x; x[1] += lo[r].y; x[2] += lo[r].z; x[3] += lo[r].w;
      x[4] += hi[r].x; x[5] += hi[r].y; x[6] += hi[r].z; x[7] += hi[r].w;
    }
    const Vec8 rr = load8(res + c);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[k][i] = x[i] + rr.v[i];
      ss += v[k][i] * v[k][i];
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (nt + 31) / 32; ++i) tot += red[i];
  const float rs = rsqrtf(tot / float(H) + eps);
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = (tid + k * nt) * 8;
    if (c >= H) break;
    store8(res + c, v[k]);
    const Vec8 wv = load8(w + c);
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      y[i] = zc ? v[k][i] * rs * (1.f + wv.v[i]) : __bfloat162float(__float2bfloat16(v[k][i] * rs)) * wv.v[i];
    if (outs == nullptr) {
      store8(out + c, y);
    } else {
      for (int r = 0; r < nout; ++r) store8(reinterpret_cast<__nv_bfloat16*>(outs[r]) + acc_row * H + c, y);
    }
  }
}

__global__ void __launch_bounds__(512) acc_norm_tp_kernel(const unsigned long long* __restrict__ accs,
                                                          float* __restrict__ my_other,
                                                          __nv_bfloat16* __restrict__ residual,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ out, int rows, int H, float eps,
                                                          bool zc, const unsigned long long* flags,
                                                          const unsigned int* my_flag, int world,
                                                          unsigned int* rows_used, int parity) {
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, row = blockIdx.x, nt = blockDim.x;
  const bool ok = wait_all_ranks(flags, my_flag, world);
  // re-zero the accumulator rows of the previous call (other parity); peers are done with them
  const int prev_rows = int(rows_used[parity ^ 1]);
  for (int r = row; r < prev_rows; r += gridDim.x)
    for (int c = tid * 4; c < H; c += nt * 4) *reinterpret_cast<float4*>(my_other + size_t(r) * H + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  if (row < rows)
    pull_add_norm_row(accs, world, ok, size_t(row), residual + size_t(row) * H, w, out + size_t(row) * H, H, eps, zc);
  if (row == 0 && tid == 0) rows_used[parity] = unsigned(rows);
}

// Every CTA makes its writes visible system-wide and counts itself in; the last one resets the
// counter and releases ``*ready += 1`` at system scope.
__device__ __forceinline__ void finish_and_release(unsigned int* done_ctr, unsigned int* ready) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(done_ctr, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(done_ctr, 0u);
      __threadfence_system();
      asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(ready) : "memory");
    }
  }
}

// Token-sharded (sequence-parallel) reduce-scatter + residual + RMSNorm + all-gather: rank r
// owns rows [row_base, row_base + rows) of the T tokens.  Each CTA pulls one of those rows from
// every rank's fp32 partial product (after every rank's row-parallel GEMM counter has caught up
// with this rank's), adds the shard's residual row, and pushes the normalised row into row
// (row_base + row) of every rank's full activation buffer (``xf``, peer memory), so each remote
// row crosses NVLink once; peers' GEMMs read it from their own memory once ``*ready`` has moved on.
__global__ void __launch_bounds__(512) sp_rs_norm_kernel(const unsigned long long* __restrict__ accs,
                                                         const unsigned long long* gflags,
                                                         const unsigned int* my_gflag, int world,
                                                         __nv_bfloat16* __restrict__ residual,
                                                         const __nv_bfloat16* __restrict__ w,
                                                         const unsigned long long* __restrict__ xf, int rows,
                                                         int row_base, int H, float eps, bool zc,
                                                         unsigned int* done_ctr, unsigned int* ready) {
  pdl_trigger();
  pdl_wait();
  const bool ok = wait_all_ranks(gflags, my_gflag, world);
  const int row = blockIdx.x;
  if (row < rows)
    pull_add_norm_row(accs, world, ok, size_t(row_base + row), residual + size_t(row) * H, w, nullptr, H, eps, zc,
                      xf, world);
  finish_and_release(done_ctr, ready);
}

// Push this rank's first normalised shard (embedding + first RMSNorm) into rows
// [row_base, row_base + rows) of every rank's full activation buffer and release ``*ready``.
__global__ void __launch_bounds__(256) sp_publish_kernel(const __nv_bfloat16* __restrict__ x,
                                                         const unsigned long long* __restrict__ xf, int world,
                                                         int rows, int row_base, int H, unsigned int* done_ctr,
                                                         unsigned int* ready) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  if (row < rows)
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + size_t(row) * H + c);
      for (int r = 0; r < world; ++r)
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(xf[r]) + size_t(row_base + row) * H + c) = v;
    }
  finish_and_release(done_ctr, ready);
}

// out[t] = row t of this rank's full activation buffer, once its owner (t / S) has pushed it
// (the owner's counter has reached this rank's).
__global__ void __launch_bounds__(256) sp_gather_kernel(const __nv_bfloat16* __restrict__ xf,
                                                        const unsigned long long* flags, const unsigned int* my_flag,
                                                        int S, int H, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  __shared__ int ok;
  const int t = blockIdx.x, owner = t / S;
  if (threadIdx.x == 0) {
    const unsigned int target = ld_acquire_sys(my_flag);
    ok = wait_counters(flags + owner, 1, target) ? 1 : 0;
  }
  __syncthreads();
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (ok) v = __ldcv(reinterpret_cast<const uint4*>(xf + size_t(t) * H + c));
    *reinterpret_cast<uint4*>(out + size_t(t) * H + c) = v;
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

at::Tensor add_rmsnorm_acc_tp(const at::Tensor& accs, at::Tensor my_acc_other, at::Tensor residual,
                              const at::Tensor& w, double eps, bool zc, const at::Tensor& flags,
                              const at::Tensor& my_flag, at::Tensor rows_used, int64_t parity) {
  TORCH_CHECK(accs.scalar_type() == at::kLong && flags.scalar_type() == at::kLong && accs.numel() == flags.numel(),
              "accs / flags must be int64 device tables of equal length");
  TORCH_CHECK(my_acc_other.scalar_type() == at::kFloat && my_acc_other.is_contiguous(), "fp32 accumulator");
  TORCH_CHECK(residual.is_contiguous() && residual.scalar_type() == at::kBFloat16, "residual must be bf16");
  TORCH_CHECK(my_flag.scalar_type() == at::kInt && rows_used.scalar_type() == at::kInt && rows_used.numel() == 2,
              "int32 flag / row-count words");
  const int H = residual.size(-1), rows = residual.numel() / H;
  TORCH_CHECK(H % 8 == 0 && H <= 16384, "hidden size must be a multiple of 8 and at most 16384");
  at::Tensor out = at::empty_like(residual);
  TORCH_CHECK(flags.numel() <= kMaxWorld, "at most ", kMaxWorld, " ranks");
  const int threads = std::min(512, ((H / 8 + 31) / 32) * 32);
  launch_pdl(acc_norm_tp_kernel, dim3(std::max(rows, 1)), dim3(threads), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const unsigned long long*>(accs.data_ptr<int64_t>()), my_acc_other.data_ptr<float>(),
             reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, H, float(eps), zc,
             reinterpret_cast<const unsigned long long*>(flags.data_ptr<int64_t>()),
             reinterpret_cast<const unsigned int*>(my_flag.data_ptr<int>()), int(flags.numel()),
             reinterpret_cast<unsigned int*>(rows_used.data_ptr<int>()), int(parity));
  return out;
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

// ---------------------------------------------------------------- sequence-parallel (token-sharded) path
// ``xf``: int64 [W] device addresses of every rank's full activation buffer (>= row_base + rows
// rows of H bf16 each; the caller sizes them).
void sp_rs_norm(const at::Tensor& accs, const at::Tensor& gflags, const at::Tensor& my_gflag, at::Tensor residual,
                const at::Tensor& w, const at::Tensor& xf, int64_t row_base, double eps, bool zc, at::Tensor done_ctr,
                at::Tensor ready) {
  TORCH_CHECK(residual.is_contiguous() && residual.scalar_type() == at::kBFloat16 && residual.dim() == 2,
              "residual shard: contiguous bf16 [rows, H]");
  const int rows = residual.size(0), H = residual.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 16384, "hidden size must be a multiple of 8 and at most 16384");
  TORCH_CHECK(gflags.numel() <= kMaxWorld && accs.numel() == gflags.numel() && xf.numel() == gflags.numel(),
              "one accumulator, counter and activation buffer per rank");
  const int threads = std::min(512, ((H / 8 + 31) / 32) * 32);
  launch_pdl(sp_rs_norm_kernel, dim3(std::max(rows, 1)), dim3(threads), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const unsigned long long*>(accs.data_ptr<int64_t>()),
             reinterpret_cast<const unsigned long long*>(gflags.data_ptr<int64_t>()),
             reinterpret_cast<const unsigned int*>(my_gflag.data_ptr<int>()), int(gflags.numel()),
             reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
             reinterpret_cast<const unsigned long long*>(xf.data_ptr<int64_t>()), rows, int(row_base), H, float(eps), zc,
             reinterpret_cast<unsigned int*>(done_ctr.data_ptr<int>()), reinterpret_cast<unsigned int*>(ready.data_ptr<int>()));
}

void sp_publish(const at::Tensor& x, const at::Tensor& xf, int64_t row_base, at::Tensor done_ctr, at::Tensor ready) {
  TORCH_CHECK(x.is_contiguous() && x.scalar_type() == at::kBFloat16 && x.dim() == 2, "x: contiguous bf16 [rows, H]");
  const int rows = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && xf.numel() <= kMaxWorld, "hidden size a multiple of 8, at most 8 ranks");
  launch_pdl(sp_publish_kernel, dim3(std::max(rows, 1)), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
             reinterpret_cast<const unsigned long long*>(xf.data_ptr<int64_t>()), int(xf.numel()), rows, int(row_base),
             H, reinterpret_cast<unsigned int*>(done_ctr.data_ptr<int>()), reinterpret_cast<unsigned int*>(ready.data_ptr<int>()));
}

at::Tensor sp_gather(const at::Tensor& xf_local, const at::Tensor& flags, const at::Tensor& my_flag, int64_t S,
                     int64_t T) {
  TORCH_CHECK(xf_local.is_contiguous() && xf_local.scalar_type() == at::kBFloat16 && xf_local.dim() == 2 &&
                  xf_local.size(0) >= T, "local activation buffer [>= T, H] bf16");
  const int64_t H = xf_local.size(1);
  TORCH_CHECK(H % 8 == 0 && S > 0 && T <= S * flags.numel(), "gather shape");
  at::Tensor out = at::empty({T, H}, xf_local.options());
  if (T == 0) return out;
  launch_pdl(sp_gather_kernel, dim3(T), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
             reinterpret_cast<const __nv_bfloat16*>(xf_local.data_ptr()),
             reinterpret_cast<const unsigned long long*>(flags.data_ptr<int64_t>()),
             reinterpret_cast<const unsigned int*>(my_flag.data_ptr<int>()), int(S), int(H),
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  return out;
}

int64_t comm_error_word() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_comm_err, sizeof(v));
  const unsigned int z = 0;
  cudaMemcpyToSymbol(g_comm_err, &z, sizeof(z));
  return v;
}

}  // namespace isb
