// Small state-maintenance kernels: int8 checkpoint quantisation (one fp32 scale per
// row of the value dimension, as in ``nanovllm/engine/state_manager.py:421-451``) and
// partial-page KV copy-on-write (``nanovllm/engine/model_runner.py:1015-1052``).

#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace isb {

namespace {

// one warp per row of ``cols`` fp32 values
__global__ void quant_rows_kernel(const float* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scale,
                                  int rows, int cols) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* r = x + size_t(row) * cols;
  float m = 0.f;
  for (int c = lane; c < cols; c += 32) m = fmaxf(m, fabsf(r[c]));
  m = warp_max(m);
  const float s = fmaxf(m / 127.f, 1e-8f);
  for (int c = lane; c < cols; c += 32) {
    const float v = rintf(r[c] / s);
    q[size_t(row) * cols + c] = int8_t(fminf(fmaxf(v, -127.f), 127.f));
  }
  if (lane == 0) scale[row] = s;
}

__global__ void dequant_rows_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                    float* __restrict__ out, int rows, int cols) {
  const size_t n = size_t(rows) * cols;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    out[i] = float(q[i]) * scale[i / cols];
}

// grid (Hkv, 2): copy rows [0, n) of page src into page dst for K (y=0) and V (y=1)
__global__ void copy_page_kernel(__nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, int Hkv, int page,
                                 int hd, int src, int dst, int n) {
  __nv_bfloat16* base = blockIdx.y == 0 ? kc : vc;
  const int h = blockIdx.x;
  const uint4* s = reinterpret_cast<const uint4*>(base + (size_t(src) * Hkv + h) * page * hd);
  uint4* d = reinterpret_cast<uint4*>(base + (size_t(dst) * Hkv + h) * page * hd);
  const int vecs = n * hd / 8;
  for (int i = threadIdx.x; i < vecs; i += blockDim.x) d[i] = s[i];
}

}  // namespace

void quantize_state_int8(const at::Tensor& state, at::Tensor q, at::Tensor scale) {
  at::Tensor x = state.to(at::kFloat).contiguous();
  TORCH_CHECK(q.is_contiguous() && q.scalar_type() == at::kChar && q.numel() == x.numel(), "int8 output mismatch");
  TORCH_CHECK(scale.is_contiguous() && scale.scalar_type() == at::kFloat, "scale must be fp32");
  const int cols = x.size(-1), rows = x.numel() / cols;
  TORCH_CHECK(scale.numel() == rows, "one scale per row");
  if (rows == 0) return;
  quant_rows_kernel<<<(rows + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), q.data_ptr<int8_t>(), scale.data_ptr<float>(), rows, cols);
}

void dequantize_state_int8(const at::Tensor& q, const at::Tensor& scale, at::Tensor out) {
  TORCH_CHECK(q.is_contiguous() && scale.is_contiguous(), "contiguous inputs");
  const int cols = q.size(-1), rows = q.numel() / cols;
  if (rows == 0) return;
  at::Tensor o = out.is_contiguous() && out.scalar_type() == at::kFloat ? out : at::empty(q.sizes(), out.options().dtype(at::kFloat));
  const int blocks = std::min<int64_t>((q.numel() + 255) / 256, 4096);
  dequant_rows_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      q.data_ptr<int8_t>(), scale.data_ptr<float>(), o.data_ptr<float>(), rows, cols);
  if (!o.is_same(out)) out.copy_(o);
}

void copy_kv_page(at::Tensor kc, at::Tensor vc, int64_t src, int64_t dst, int64_t n) {
  TORCH_CHECK(kc.dim() == 4 && kc.is_contiguous() && vc.is_contiguous(), "KV cache must be [blocks, Hkv, page, hd]");
  const int Hkv = kc.size(1), page = kc.size(2), hd = kc.size(3);
  TORCH_CHECK(n >= 0 && n <= page && src >= 0 && dst >= 0 && src < kc.size(0) && dst < kc.size(0), "bad page copy");
  if (n == 0) return;
  copy_page_kernel<<<dim3(Hkv, 2), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(kc.data_ptr()), reinterpret_cast<__nv_bfloat16*>(vc.data_ptr()), Hkv, page, hd,
      int(src), int(dst), int(n));
}

}  // namespace isb
