// RMSNorm family and embedding lookup (memory-bound; one warp per row, 16-byte vectors).
//
// rmsnorm:      out = x * rsqrt(mean(x^2) + eps) * (1 + w)   (zero-centred, Qwen3.5)
//                     bf16(x * rsqrt(..)) * w                 (plain, Qwen3)
// add_rmsnorm:  s = x + residual (fp32); residual <- bf16(s); out = norm(s) of the
//               UNROUNDED sum -- the rounding order of the reference's fused
//               add+norm (``nanovllm/csrc/fused_add_rmsnorm_kernel.cu:81-153``).
// embed_rmsnorm: residual <- embedding rows; out = norm(residual) (first layer).

#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"

namespace isb {

namespace {

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

__device__ __forceinline__ void norm_store8(__nv_bfloat16* o, const float* s, const __nv_bfloat16* w, float rs,
                                            bool zc) {
  const Vec8 wv = load8(w);
  float y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (zc) {
      y[i] = s[i] * rs * (1.0f + wv.v[i]);
    } else {
      y[i] = __bfloat162float(__float2bfloat16(s[i] * rs)) * wv.v[i];
    }
  }
  store8(o, y);
}

// MODE 0: rmsnorm(x); MODE 1: add_rmsnorm(x, residual); MODE 2: embedding gather + rmsnorm
template <int MODE>
__global__ void norm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                            const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                            const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int rows, int H,
                            float eps, bool zc) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* src = nullptr;
  if constexpr (MODE == 2) src = table + size_t(ids[row]) * H;
  else src = x + size_t(row) * H;
  __nv_bfloat16* res = MODE == 1 || MODE == 2 ? residual + size_t(row) * H : nullptr;
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    Vec8 a = load8(src + c);
    if constexpr (MODE == 1) {
      const Vec8 r = load8(res + c);
#pragma unroll
      for (int i = 0; i < 8; ++i) a.v[i] += r.v[i];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += a.v[i] * a.v[i];
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / float(H) + eps);
  for (int c = lane * 8; c < H; c += 256) {
    Vec8 a = load8(src + c);
    if constexpr (MODE == 1) {
      const Vec8 r = load8(res + c);
#pragma unroll
      for (int i = 0; i < 8; ++i) a.v[i] += r.v[i];
    }
    if constexpr (MODE == 1 || MODE == 2) store8(res + c, a.v);
    norm_store8(out + size_t(row) * H + c, a.v, w + c, rs, zc);
  }
}

__global__ void embed_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             __nv_bfloat16* __restrict__ out, int rows, int H, int vocab_start, int vocab_rows) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int id = ids[row] - vocab_start;
  const bool ok = id >= 0 && id < vocab_rows;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (ok) v = *reinterpret_cast<const uint4*>(table + size_t(id) * H + c);
    *reinterpret_cast<uint4*>(out + size_t(row) * H + c) = v;
  }
}

constexpr int kRowsPerBlock = 4;

void check_rows(const at::Tensor& x, const at::Tensor& w) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "expected contiguous bf16 CUDA rows");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.numel() == x.size(-1), "norm weight mismatch");
  TORCH_CHECK(x.size(-1) % 8 == 0, "hidden size must be a multiple of 8");
}

}  // namespace

at::Tensor rmsnorm(const at::Tensor& x_in, const at::Tensor& w, double eps, bool zc) {
  at::Tensor x = x_in.contiguous();
  check_rows(x, w);
  at::Tensor out = at::empty_like(x);
  const int H = x.size(-1), rows = x.numel() / H;
  if (rows == 0) return out;
  norm_kernel<0><<<(rows + kRowsPerBlock - 1) / kRowsPerBlock, 32 * kRowsPerBlock, 0,
                   at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), nullptr, nullptr, nullptr,
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, H,
      float(eps), zc);
  return out;
}

at::Tensor add_rmsnorm(const at::Tensor& x_in, at::Tensor residual, const at::Tensor& w, double eps, bool zc) {
  at::Tensor x = x_in.contiguous();
  check_rows(x, w);
  TORCH_CHECK(residual.is_contiguous() && residual.sizes() == x.sizes() && residual.scalar_type() == x.scalar_type(),
              "residual must match x");
  at::Tensor out = at::empty_like(x);
  const int H = x.size(-1), rows = x.numel() / H;
  if (rows == 0) return out;
  norm_kernel<1><<<(rows + kRowsPerBlock - 1) / kRowsPerBlock, 32 * kRowsPerBlock, 0,
                   at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()),
      nullptr, nullptr, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, H, float(eps), zc);
  return out;
}

std::tuple<at::Tensor, at::Tensor> embed_rmsnorm(const at::Tensor& ids, const at::Tensor& table, const at::Tensor& w,
                                                 double eps, bool zc) {
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "ids must be contiguous int32");
  TORCH_CHECK(table.scalar_type() == at::kBFloat16 && table.is_contiguous(), "embedding table must be bf16");
  const int rows = ids.numel(), H = table.size(1);
  at::Tensor residual = at::empty({rows, H}, table.options());
  at::Tensor out = at::empty({rows, H}, table.options());
  if (rows == 0) return {residual, out};
  norm_kernel<2><<<(rows + kRowsPerBlock - 1) / kRowsPerBlock, 32 * kRowsPerBlock, 0,
                   at::cuda::getCurrentCUDAStream()>>>(
      nullptr, reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()), ids.data_ptr<int>(),
      reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, H, float(eps), zc);
  return {residual, out};
}

at::Tensor embed(const at::Tensor& ids, const at::Tensor& table, int64_t vocab_start) {
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "ids must be contiguous int32");
  TORCH_CHECK(table.scalar_type() == at::kBFloat16 && table.is_contiguous() && table.size(1) % 8 == 0,
              "embedding table must be contiguous bf16 with H % 8 == 0");
  const int rows = ids.numel(), H = table.size(1);
  at::Tensor out = at::empty({rows, H}, table.options());
  if (rows == 0) return out;
  embed_kernel<<<(rows + kRowsPerBlock - 1) / kRowsPerBlock, 32 * kRowsPerBlock, 0,
                 at::cuda::getCurrentCUDAStream()>>>(ids.data_ptr<int>(),
                                                     reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
                                                     reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, H,
                                                     int(vocab_start), int(table.size(0)));
  return out;
}

}  // namespace isb
