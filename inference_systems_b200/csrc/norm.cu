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
#include "launch.cuh"

namespace isb {

namespace {

// MODE 3: s = acc (fp32) + residual; residual <- bf16(s); out = norm(s); acc <- 0
__global__ void acc_norm_kernel(float* __restrict__ acc, __nv_bfloat16* __restrict__ residual,
                                const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int rows, int H,
                                float eps, bool zc) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float* a = acc + size_t(row) * H;
  __nv_bfloat16* res = residual + size_t(row) * H;
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    const float4 x0 = *reinterpret_cast<const float4*>(a + c), x1 = *reinterpret_cast<const float4*>(a + c + 4);
    const Vec8 r = load8(res + c);
    const float v[8] = {x0.x + r.v[0], x0.y + r.v[1], x0.z + r.v[2], x0.w + r.v[3],
                        x1.x + r.v[4], x1.y + r.v[5], x1.z + r.v[6], x1.w + r.v[7]};
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / float(H) + eps);
  for (int c = lane * 8; c < H; c += 256) {
    const float4 x0 = *reinterpret_cast<const float4*>(a + c), x1 = *reinterpret_cast<const float4*>(a + c + 4);
    const Vec8 r = load8(res + c);
    float v[8] = {x0.x + r.v[0], x0.y + r.v[1], x0.z + r.v[2], x0.w + r.v[3],
                  x1.x + r.v[4], x1.y + r.v[5], x1.z + r.v[6], x1.w + r.v[7]};
    store8(res + c, v);
    norm_store8(out + size_t(row) * H + c, v, w + c, rs, zc);
    *reinterpret_cast<float4*>(a + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(a + c + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// MODE 0: rmsnorm(x); MODE 1: add_rmsnorm(x, residual); MODE 2: embedding gather + rmsnorm
template <int MODE>
__global__ void norm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                            const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                            const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int rows, int H,
                            float eps, bool zc) {
  pdl_trigger();
  pdl_wait();
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
  pdl_trigger();
  pdl_wait();
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
  launch_pdl(norm_kernel<0>, dim3((rows + kRowsPerBlock - 1) / kRowsPerBlock), dim3(32 * kRowsPerBlock), 0, at::cuda::getCurrentCUDAStream(), 
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
  launch_pdl(norm_kernel<1>, dim3((rows + kRowsPerBlock - 1) / kRowsPerBlock), dim3(32 * kRowsPerBlock), 0, at::cuda::getCurrentCUDAStream(), 
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()),
      nullptr, nullptr, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, H, float(eps), zc);
  return out;
}

// out[t, g*64 + j] = SiLU(acc[t, g*128 + j]) * acc[t, g*128 + 64 + j]  (packed gate/up groups of 64), acc <- 0
__global__ void silu_mul_acc_kernel(float* __restrict__ acc, __nv_bfloat16* __restrict__ out, int rows, int inter) {
  pdl_trigger();
  pdl_wait();
  const int groups4 = inter / 4;  // output vectors of 4 per row
  const size_t n = size_t(rows) * groups4;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const int t = int(i / groups4), o = int(i % groups4) * 4;
    const int g = o / 64, j = o % 64;
    float* base = acc + size_t(t) * 2 * inter + g * 128 + j;
    const float4 gv = *reinterpret_cast<const float4*>(base);
    const float4 uv = *reinterpret_cast<const float4*>(base + 64);
    *reinterpret_cast<float4*>(base) = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(base + 64) = make_float4(0.f, 0.f, 0.f, 0.f);
    __nv_bfloat162 lo = __floats2bfloat162_rn(silu(gv.x) * uv.x, silu(gv.y) * uv.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(silu(gv.z) * uv.z, silu(gv.w) * uv.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&lo);
    pk.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(out + size_t(t) * inter + o) = pk;
  }
}

at::Tensor silu_mul_acc(at::Tensor acc, int64_t rows) {
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.dim() == 2, "fp32 [rows, 2I] accumulator");
  const int inter = acc.size(1) / 2;
  TORCH_CHECK(inter % 64 == 0 && rows <= acc.size(0), "intermediate size must be a multiple of 64");
  at::Tensor out = at::empty({rows, inter}, acc.options().dtype(at::kBFloat16));
  if (rows == 0) return out;
  const size_t n = size_t(rows) * inter / 4;
  const int blocks = int(std::min<size_t>((n + 255) / 256, 148 * 8));
  launch_pdl(silu_mul_acc_kernel, dim3(blocks), dim3(256), 0, at::cuda::getCurrentCUDAStream(), 
      acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(rows), inter);
  return out;
}

at::Tensor add_rmsnorm_acc(at::Tensor acc, at::Tensor residual, const at::Tensor& w, double eps, bool zc) {
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous(), "accumulator must be contiguous fp32");
  check_rows(residual, w);
  const int H = residual.size(-1), rows = residual.numel() / H;
  TORCH_CHECK(acc.size(-1) == H && acc.numel() >= size_t(rows) * H, "accumulator shape mismatch");
  at::Tensor out = at::empty_like(residual);
  if (rows == 0) return out;
  launch_pdl(acc_norm_kernel, dim3((rows + kRowsPerBlock - 1) / kRowsPerBlock), dim3(32 * kRowsPerBlock), 0, at::cuda::getCurrentCUDAStream(), acc.data_ptr<float>(),
                                                        reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()),
                                                        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                                                        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, H,
                                                        float(eps), zc);
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
  launch_pdl(norm_kernel<2>, dim3((rows + kRowsPerBlock - 1) / kRowsPerBlock), dim3(32 * kRowsPerBlock), 0, at::cuda::getCurrentCUDAStream(), 
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
  launch_pdl(embed_kernel, dim3((rows + kRowsPerBlock - 1) / kRowsPerBlock), dim3(32 * kRowsPerBlock), 0, at::cuda::getCurrentCUDAStream(), ids.data_ptr<int>(),
                                                     reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
                                                     reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, H,
                                                     int(vocab_start), int(table.size(0)));
  return out;
}

}  // namespace isb
