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

// One block of 128 threads per row (8 columns per thread per step).
__global__ void __launch_bounds__(128) acc_norm_tp_kernel(const unsigned long long* __restrict__ accs,
                                                          float* __restrict__ my_other,
                                                          __nv_bfloat16* __restrict__ residual,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ out, int rows, int H, float eps,
                                                          bool zc, const unsigned long long* flags,
                                                          const unsigned int* my_flag, int world,
                                                          unsigned int* rows_used, int parity) {
  pdl_trigger();
  pdl_wait();
  __shared__ int ok;
  __shared__ float red[4];
  const int tid = threadIdx.x, row = blockIdx.x;
  if (tid == 0) ok = 1;
  __syncthreads();
  if (tid < world) {  // every peer's counter is polled by its own thread: one NVLink round trip, not world
    const unsigned int target = ld_acquire_sys(my_flag);  // this rank's GEMM of this call has completed
    if (!wait_counters(flags + tid, 1, target)) ok = 0;
  }
  __syncthreads();
  // re-zero the accumulator rows of the previous call (other parity); peers are done with them
  const int prev_rows = int(rows_used[parity ^ 1]);
  for (int r = row; r < prev_rows; r += gridDim.x)
    for (int c = tid * 4; c < H; c += 512) *reinterpret_cast<float4*>(my_other + size_t(r) * H + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  if (row < rows) {
    __nv_bfloat16* res = residual + size_t(row) * H;
    float ss = 0.f;
    constexpr int kMaxChunks = 8;  // H <= 8 * 1024
    float v[kMaxChunks][8];
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = tid * 8 + k * 1024;
      if (c >= H) break;
      float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (ok) {
        for (int r = 0; r < world; ++r) {
          const float* a = reinterpret_cast<const float*>(accs[r]) + size_t(row) * H + c;
          const float4 x0 = __ldcv(reinterpret_cast<const float4*>(a));
          const float4 x1 = __ldcv(reinterpret_cast<const float4*>(a + 4));
          x[0] += x0.x; x[1] += x0.y; x[2] += x0.z; x[3] += x0.w;
          x[4] += x1.x; x[5] += x1.y; x[6] += x1.z; x[7] += x1.w;
        }
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
    const float rs = rsqrtf((red[0] + red[1] + red[2] + red[3]) / float(H) + eps);
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = tid * 8 + k * 1024;
      if (c >= H) break;
      store8(res + c, v[k]);
      const Vec8 wv = load8(w + c);
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        y[i] = zc ? v[k][i] * rs * (1.f + wv.v[i]) : __bfloat162float(__float2bfloat16(v[k][i] * rs)) * wv.v[i];
      store8(out + size_t(row) * H + c, y);
    }
  }
  if (row == 0 && tid == 0) rows_used[parity] = unsigned(rows);
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
  TORCH_CHECK(H % 8 == 0 && H <= 8192, "hidden size must be a multiple of 8 and at most 8192");
  at::Tensor out = at::empty_like(residual);
  launch_pdl(acc_norm_tp_kernel, dim3(std::max(rows, 1)), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
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

int64_t comm_error_word() {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_comm_err, sizeof(v));
  const unsigned int z = 0;
  cudaMemcpyToSymbol(g_comm_err, &z, sizeof(z));
  return v;
}

}  // namespace isb
