// Fused residual-add + RMSNorm, plain RMSNorm and LayerNorm (fwd + bwd).
//
// One CTA of 256 threads owns a row at a time and walks rows with a grid
// stride; each thread keeps its 8*NCH elements in registers (vectorised 16-byte
// loads).  Weight gradients are reduced per CTA in registers (over all of the
// CTA's rows), written as one row per CTA of a small [CTAs, H] buffer, and
// summed into the gradient by ``colsum_add_kernel`` -- deterministic and free
// of same-address atomics (the reference's Triton kernel wrote a [rows, H]
// partial buffer instead, kernels/rmsnorm.py:43-104).
#include "common.cuh"
#include "tmap.h"

namespace nq {

constexpr int kNormThreads = 256;

template <typename T> __device__ __forceinline__ void ld8(const T* p, float (&f)[8]) { load8(p, f); }
template <typename T> __device__ __forceinline__ void st8(T* p, const float (&f)[8]) { store8(p, f); }

// h = resid (+ delta); y = bf16(h * rstd * w)
template <int NCH>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_fwd_kernel(
    const float* __restrict__ resid, const __nv_bfloat16* __restrict__ delta,
    const float* __restrict__ w, float* __restrict__ h_out, __nv_bfloat16* __restrict__ y,
    float* __restrict__ rstd_out, int T, int H, float eps) {
  __shared__ float red[32];
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    float v[NCH][8];
    float ss = 0.f;
    const int64_t base = static_cast<int64_t>(row) * H;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        ld8(resid + base + col, v[c]);
        if (delta != nullptr) {
          float d[8];
          ld8(delta + base + col, d);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[c][i] += d[i];
        }
        st8(h_out + base + col, v[c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
      }
    }
    ss = block_sum(ss, red);
    const float r = rsqrtf(ss / H + eps);
    if (threadIdx.x == 0) rstd_out[row] = r;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        float wv[8], o[8];
        ld8(w + col, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[c][i] * r * wv[i];
        st8(y + base + col, o);
      }
    }
  }
}

// dx = dh + rstd * (g - xhat * mean(g * xhat)),  g = dy * w,  xhat = h * rstd
// dw += sum_rows dy * xhat
template <int NCH>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const float* __restrict__ dh,
    const float* __restrict__ h, const float* __restrict__ w, const float* __restrict__ rstd,
    float* __restrict__ dx, __nv_bfloat16* __restrict__ dx_bf16, float* __restrict__ dw,
    int T, int H) {
  __shared__ float red[32];
  float dwacc[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) dwacc[c][i] = 0.f;
  float wv[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * kNormThreads + threadIdx.x) * 8;
    if (col < H) ld8(w + col, wv[c]);
  }
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const int64_t base = static_cast<int64_t>(row) * H;
    const float r = rstd[row];
    float xh[NCH][8], g[NCH][8], res[NCH][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        float hv[8], d[8];
        ld8(h + base + col, hv);
        ld8(dy + base + col, d);
        // the incoming residual gradient is loaded with the row, before the
        // block reduction, so each row costs one memory round trip
        if (dh != nullptr) ld8(dh + base + col, res[c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          xh[c][i] = hv[i] * r;
          g[c][i] = d[i] * wv[c][i];
          dot += g[c][i] * xh[c][i];
          dwacc[c][i] += d[i] * xh[c][i];
        }
      }
    }
    dot = block_sum(dot, red) / H;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[i] = r * (g[c][i] - xh[c][i] * dot) + (dh != nullptr ? res[c][i] : 0.f);
        }
        st8(dx + base + col, o);
        if (dx_bf16 != nullptr) st8(dx_bf16 + base + col, o);
      }
    }
  }
  if (dw != nullptr) {  // this CTA's row of the [gridDim.x, H] partial buffer
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) st8(dw + static_cast<int64_t>(blockIdx.x) * H + col, dwacc[c]);
    }
  }
}

// Plain RMSNorm: y = (x * rstd) * w (x bf16 or fp32, y bf16 or fp32).
template <int NCH, typename TI, typename TO>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_kernel(
    const TI* __restrict__ x, const float* __restrict__ w, TO* __restrict__ y,
    float* __restrict__ rstd_out, int T, int H, float eps) {
  __shared__ float red[32];
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    float v[NCH][8];
    float ss = 0.f;
    const int64_t base = static_cast<int64_t>(row) * H;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        ld8(x + base + col, v[c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
      }
    }
    ss = block_sum(ss, red);
    const float r = rsqrtf(ss / H + eps);
    if (threadIdx.x == 0) rstd_out[row] = r;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        float wv[8], o[8];
        ld8(w + col, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[c][i] * r * wv[i];
        st8(y + base + col, o);
      }
    }
  }
}

template <int NCH, typename TI>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_bwd_kernel(
    const TI* __restrict__ dy, const TI* __restrict__ x, const float* __restrict__ w,
    const float* __restrict__ rstd, float* __restrict__ dx, float* __restrict__ dw, int T, int H) {
  __shared__ float red[32];
  float dwacc[NCH][8];
  float wv[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * kNormThreads + threadIdx.x) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) dwacc[c][i] = 0.f;
    if (col < H) ld8(w + col, wv[c]);
  }
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const int64_t base = static_cast<int64_t>(row) * H;
    const float r = rstd[row];
    float xh[NCH][8], g[NCH][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        float xv[8], d[8];
        ld8(x + base + col, xv);
        ld8(dy + base + col, d);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          xh[c][i] = xv[i] * r;
          g[c][i] = d[i] * wv[c][i];
          dot += g[c][i] * xh[c][i];
          dwacc[c][i] += d[i] * xh[c][i];
        }
      }
    }
    dot = block_sum(dot, red) / H;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = r * (g[c][i] - xh[c][i] * dot);
        st8(dx + base + col, o);
      }
    }
  }
  if (dw != nullptr) {  // this CTA's row of the [gridDim.x, H] partial buffer
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) st8(dw + static_cast<int64_t>(blockIdx.x) * H + col, dwacc[c]);
    }
  }
}

// LayerNorm: y = (x - mean) * rstd * w + b
template <int NCH, typename TI, typename TO>
__global__ void __launch_bounds__(kNormThreads) layernorm_fwd_kernel(
    const TI* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
    TO* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out, int T, int H,
    float eps) {
  __shared__ float red[32];
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    float v[NCH][8];
    float s = 0.f;
    const int64_t base = static_cast<int64_t>(row) * H;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        ld8(x + base + col, v[c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) s += v[c][i];
      }
    }
    const float mean = block_sum(s, red) / H;
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H)
#pragma unroll
        for (int i = 0; i < 8; ++i) { float d = v[c][i] - mean; ss += d * d; }
    }
    const float r = rsqrtf(block_sum(ss, red) / H + eps);
    if (threadIdx.x == 0) { rstd_out[row] = r; mean_out[row] = mean; }
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        float wv[8], bv[8], o[8];
        ld8(w + col, wv);
        if (b != nullptr) ld8(b + col, bv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = (v[c][i] - mean) * r * wv[i] + (b != nullptr ? bv[i] : 0.f);
        st8(y + base + col, o);
      }
    }
  }
}

template <int NCH, typename TI>
__global__ void __launch_bounds__(kNormThreads) layernorm_bwd_kernel(
    const TI* __restrict__ dy, const TI* __restrict__ x, const float* __restrict__ w,
    const float* __restrict__ mean, const float* __restrict__ rstd, float* __restrict__ dx,
    float* __restrict__ dw, float* __restrict__ db, int T, int H) {
  __shared__ float red[32];
  float dwacc[NCH][8], dbacc[NCH][8], wv[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * kNormThreads + threadIdx.x) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) { dwacc[c][i] = 0.f; dbacc[c][i] = 0.f; }
    if (col < H) ld8(w + col, wv[c]);
  }
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const int64_t base = static_cast<int64_t>(row) * H;
    const float r = rstd[row], mu = mean[row];
    float xh[NCH][8], g[NCH][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        float xv[8], d[8];
        ld8(x + base + col, xv);
        ld8(dy + base + col, d);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          xh[c][i] = (xv[i] - mu) * r;
          g[c][i] = d[i] * wv[c][i];
          s1 += g[c][i];
          s2 += g[c][i] * xh[c][i];
          dwacc[c][i] += d[i] * xh[c][i];
          dbacc[c][i] += d[i];
        }
      }
    }
    s1 = block_sum(s1, red) / H;
    s2 = block_sum(s2, red) / H;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kNormThreads + threadIdx.x) * 8;
      if (col < H) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = r * (g[c][i] - s1 - xh[c][i] * s2);
        st8(dx + base + col, o);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * kNormThreads + threadIdx.x) * 8;
    if (col < H) {
      if (dw != nullptr) st8(dw + static_cast<int64_t>(blockIdx.x) * H + col, dwacc[c]);
      if (db != nullptr) st8(db + static_cast<int64_t>(blockIdx.x) * H + col, dbacc[c]);
    }
  }
}

// --------------------------------------------------------------------- host
static int norm_grid(int T) { return std::max(1, std::min(T, num_sms() * 8)); }

// out[c] += sum_b part[b, c]; grid (ceil(H/32), splits), block (32, 8).
__global__ void __launch_bounds__(256) colsum_add_kernel(const float* __restrict__ part, int G, int H,
                                                         float* __restrict__ out) {
  __shared__ float red[8][33];
  const int col = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (col < H)
    for (int b = blockIdx.y * 8 + threadIdx.y; b < G; b += 8 * gridDim.y)
      s += part[static_cast<int64_t>(b) * H + col];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && col < H) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x];
    if (gridDim.y == 1) out[col] += t; else atomicAdd(out + col, t);
  }
}

// Partial weight-gradient buffer for a backward launch with `grid` CTAs.
static torch::Tensor wgrad_partial(const torch::Tensor& like, int grid, int H) {
  return torch::empty({grid, H}, like.options().dtype(torch::kFloat32));
}

static void colsum_add(const torch::Tensor& part, float* out, cudaStream_t st) {
  const int G = part.size(0), H = part.size(1);
  const int cb = (H + 31) / 32;
  const int splits = std::max(1, std::min(G / 64, (2 * num_sms() + cb - 1) / cb));
  colsum_add_kernel<<<dim3(cb, splits), dim3(32, 8), 0, st>>>(part.data_ptr<float>(), G, H, out);
  NQ_CHECK_CUDA(cudaGetLastError());
}
static int nch_for(int H) {
  TORCH_CHECK(H % 8 == 0, "norm: hidden size must be a multiple of 8");
  int n = (H / 8 + kNormThreads - 1) / kNormThreads;
  TORCH_CHECK(n <= 4, "norm: hidden size > 8192 not supported");
  return n <= 1 ? 1 : (n <= 2 ? 2 : 4);
}

#define NQ_NCH_DISPATCH(nch, ...)           \
  switch (nch) {                            \
    case 1: { constexpr int NCH = 1; __VA_ARGS__; break; } \
    case 2: { constexpr int NCH = 2; __VA_ARGS__; break; } \
    default: { constexpr int NCH = 4; __VA_ARGS__; break; } \
  }

std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor resid, c10::optional<torch::Tensor> delta,
                                           torch::Tensor w, double eps) {
  TORCH_CHECK(resid.scalar_type() == torch::kFloat32 && resid.is_contiguous(), "resid must be fp32 contiguous");
  TORCH_CHECK(w.scalar_type() == torch::kFloat32, "norm weight must be fp32");
  const int T = resid.size(0), H = resid.size(1);
  c10::cuda::CUDAGuard g(resid.device());
  auto y = torch::empty({T, H}, resid.options().dtype(torch::kBFloat16));
  auto rstd = torch::empty({T}, resid.options());
  torch::Tensor h = torch::empty_like(resid);
  const __nv_bfloat16* dptr = nullptr;
  if (delta.has_value() && delta->defined()) {
    check_bf16(*delta, "delta");
    TORCH_CHECK(delta->is_contiguous(), "delta contiguous");
    dptr = reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr());
  }
  if (T == 0) return {h, y, rstd};
  auto st = at::cuda::getCurrentCUDAStream();
  NQ_NCH_DISPATCH(nch_for(H),
    add_rmsnorm_fwd_kernel<NCH><<<norm_grid(T), kNormThreads, 0, st>>>(
        resid.data_ptr<float>(), dptr, w.data_ptr<float>(), h.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), T, H, (float)eps));
  NQ_CHECK_CUDA(cudaGetLastError());
  return {h, y, rstd};
}

std::vector<torch::Tensor> add_rmsnorm_bwd(torch::Tensor dy, c10::optional<torch::Tensor> dh,
                                           torch::Tensor h, torch::Tensor w, torch::Tensor rstd,
                                           c10::optional<torch::Tensor> dw) {
  check_bf16(dy, "dy");
  const int T = h.size(0), H = h.size(1);
  c10::cuda::CUDAGuard g(h.device());
  auto dx = torch::empty({T, H}, h.options());
  auto dxb = torch::empty({T, H}, h.options().dtype(torch::kBFloat16));
  const float* dhp = nullptr;
  if (dh.has_value() && dh->defined()) {
    TORCH_CHECK(dh->scalar_type() == torch::kFloat32 && dh->is_contiguous(), "dh fp32 contiguous");
    dhp = dh->data_ptr<float>();
  }
  float* dwp = (dw.has_value() && dw->defined()) ? dw->data_ptr<float>() : nullptr;
  if (T == 0) return {dx, dxb};
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = norm_grid(T);
  torch::Tensor part;
  if (dwp != nullptr) part = wgrad_partial(h, grid, H);
  NQ_NCH_DISPATCH(nch_for(H),
    add_rmsnorm_bwd_kernel<NCH><<<grid, kNormThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.contiguous().data_ptr()), dhp, h.data_ptr<float>(),
        w.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dxb.data_ptr()),
        dwp != nullptr ? part.data_ptr<float>() : nullptr, T, H));
  NQ_CHECK_CUDA(cudaGetLastError());
  if (dwp != nullptr) colsum_add(part, dwp, st);
  return {dx, dxb};
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps,
                                       c10::ScalarType out_dtype) {
  TORCH_CHECK(x.is_contiguous(), "x contiguous");
  const int T = x.size(0), H = x.size(1);
  c10::cuda::CUDAGuard g(x.device());
  auto y = torch::empty({T, H}, x.options().dtype(out_dtype));
  auto rstd = torch::empty({T}, x.options().dtype(torch::kFloat32));
  if (T == 0) return {y, rstd};
  auto st = at::cuda::getCurrentCUDAStream();
  const int nch = nch_for(H);
  const bool xb = x.scalar_type() == torch::kBFloat16, yb = out_dtype == torch::kBFloat16;
  NQ_NCH_DISPATCH(nch,
    if (xb && yb) rmsnorm_fwd_kernel<NCH, __nv_bfloat16, __nv_bfloat16><<<norm_grid(T), kNormThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), T, H, (float)eps);
    else if (xb) rmsnorm_fwd_kernel<NCH, __nv_bfloat16, float><<<norm_grid(T), kNormThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr<float>(), y.data_ptr<float>(), rstd.data_ptr<float>(), T, H, (float)eps);
    else if (yb) rmsnorm_fwd_kernel<NCH, float, __nv_bfloat16><<<norm_grid(T), kNormThreads, 0, st>>>(
        x.data_ptr<float>(), w.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), T, H, (float)eps);
    else rmsnorm_fwd_kernel<NCH, float, float><<<norm_grid(T), kNormThreads, 0, st>>>(
        x.data_ptr<float>(), w.data_ptr<float>(), y.data_ptr<float>(), rstd.data_ptr<float>(), T, H, (float)eps));
  NQ_CHECK_CUDA(cudaGetLastError());
  return {y, rstd};
}

torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd,
                          c10::optional<torch::Tensor> dw) {
  const int T = x.size(0), H = x.size(1);
  c10::cuda::CUDAGuard g(x.device());
  auto dx = torch::empty({T, H}, x.options().dtype(torch::kFloat32));
  float* dwp = (dw.has_value() && dw->defined()) ? dw->data_ptr<float>() : nullptr;
  if (T == 0) return dx;
  auto dyc = dy.to(x.scalar_type()).contiguous();
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = norm_grid(T);
  torch::Tensor part;
  if (dwp != nullptr) part = wgrad_partial(x, grid, H);
  float* pp = dwp != nullptr ? part.data_ptr<float>() : nullptr;
  NQ_NCH_DISPATCH(nch_for(H),
    if (x.scalar_type() == torch::kBFloat16)
      rmsnorm_bwd_kernel<NCH, __nv_bfloat16><<<grid, kNormThreads, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(dyc.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
          w.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr<float>(), pp, T, H);
    else
      rmsnorm_bwd_kernel<NCH, float><<<grid, kNormThreads, 0, st>>>(
          dyc.data_ptr<float>(), x.data_ptr<float>(), w.data_ptr<float>(), rstd.data_ptr<float>(),
          dx.data_ptr<float>(), pp, T, H));
  NQ_CHECK_CUDA(cudaGetLastError());
  if (dwp != nullptr) colsum_add(part, dwp, st);
  return dx;
}

std::vector<torch::Tensor> layernorm_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b,
                                         double eps, c10::ScalarType out_dtype) {
  TORCH_CHECK(x.is_contiguous(), "x contiguous");
  const int T = x.size(0), H = x.size(1);
  c10::cuda::CUDAGuard g(x.device());
  auto y = torch::empty({T, H}, x.options().dtype(out_dtype));
  auto mean = torch::empty({T}, x.options().dtype(torch::kFloat32));
  auto rstd = torch::empty({T}, x.options().dtype(torch::kFloat32));
  if (T == 0) return {y, mean, rstd};
  const float* bp = (b.has_value() && b->defined()) ? b->data_ptr<float>() : nullptr;
  auto st = at::cuda::getCurrentCUDAStream();
  const bool xb = x.scalar_type() == torch::kBFloat16, yb = out_dtype == torch::kBFloat16;
  NQ_NCH_DISPATCH(nch_for(H),
    if (xb && yb) layernorm_fwd_kernel<NCH, __nv_bfloat16, __nv_bfloat16><<<norm_grid(T), kNormThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr<float>(), bp, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), mean.data_ptr<float>(), rstd.data_ptr<float>(), T, H, (float)eps);
    else if (xb) layernorm_fwd_kernel<NCH, __nv_bfloat16, float><<<norm_grid(T), kNormThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr<float>(), bp, y.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(), T, H, (float)eps);
    else if (yb) layernorm_fwd_kernel<NCH, float, __nv_bfloat16><<<norm_grid(T), kNormThreads, 0, st>>>(
        x.data_ptr<float>(), w.data_ptr<float>(), bp, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), mean.data_ptr<float>(), rstd.data_ptr<float>(), T, H, (float)eps);
    else layernorm_fwd_kernel<NCH, float, float><<<norm_grid(T), kNormThreads, 0, st>>>(
        x.data_ptr<float>(), w.data_ptr<float>(), bp, y.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(), T, H, (float)eps));
  NQ_CHECK_CUDA(cudaGetLastError());
  return {y, mean, rstd};
}

torch::Tensor layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean,
                            torch::Tensor rstd, c10::optional<torch::Tensor> dw,
                            c10::optional<torch::Tensor> db) {
  const int T = x.size(0), H = x.size(1);
  c10::cuda::CUDAGuard g(x.device());
  auto dx = torch::empty({T, H}, x.options().dtype(torch::kFloat32));
  if (T == 0) return dx;
  float* dwp = (dw.has_value() && dw->defined()) ? dw->data_ptr<float>() : nullptr;
  float* dbp = (db.has_value() && db->defined()) ? db->data_ptr<float>() : nullptr;
  auto dyc = dy.to(x.scalar_type()).contiguous();
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = norm_grid(T);
  torch::Tensor pw, pb;
  if (dwp != nullptr) pw = wgrad_partial(x, grid, H);
  if (dbp != nullptr) pb = wgrad_partial(x, grid, H);
  float* pwp = dwp != nullptr ? pw.data_ptr<float>() : nullptr;
  float* pbp = dbp != nullptr ? pb.data_ptr<float>() : nullptr;
  NQ_NCH_DISPATCH(nch_for(H),
    if (x.scalar_type() == torch::kBFloat16)
      layernorm_bwd_kernel<NCH, __nv_bfloat16><<<grid, kNormThreads, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(dyc.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
          w.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr<float>(), pwp, pbp, T, H);
    else
      layernorm_bwd_kernel<NCH, float><<<grid, kNormThreads, 0, st>>>(
          dyc.data_ptr<float>(), x.data_ptr<float>(), w.data_ptr<float>(), mean.data_ptr<float>(),
          rstd.data_ptr<float>(), dx.data_ptr<float>(), pwp, pbp, T, H));
  NQ_CHECK_CUDA(cudaGetLastError());
  if (dwp != nullptr) colsum_add(pw, dwp, st);
  if (dbp != nullptr) colsum_add(pb, dbp, st);
  return dx;
}

}  // namespace nq
