// Bandwidth-bound kernels: SwiGLU, GELU, scaling, embedding gather/scatter,
// the vocab-chunked cross-entropy row kernels, grad-norm and the flat AdamW.
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace nq {

// ------------------------------------------------------------- error word
// Default wait limits: 2 s for mbarrier waits inside one CTA (a pipeline stage
// that has not arrived by then never will), 20 s for flags written by another
// GPU (ranks can be far apart at start-up, e.g. one still compiling or loading).
constexpr uint64_t kDefaultMbarLimitNs = 2000000000ull;
constexpr uint64_t kDefaultPeerLimitNs = 20000000000ull;

int* error_flag_ptr() {
  static std::mutex mu;
  static int* block[kMaxDevices] = {};
  static torch::Tensor owner[kMaxDevices];
  const int dev = current_device();
  if (block[dev] != nullptr) return block[dev];
  std::lock_guard<std::mutex> lk(mu);
  if (block[dev] == nullptr) {
    auto t = torch::zeros({8}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, dev));
    const uint64_t lim[2] = {kDefaultMbarLimitNs, kDefaultPeerLimitNs};
    NQ_CHECK_CUDA(cudaMemcpy(t.data_ptr<int>() + 2, lim, sizeof(lim), cudaMemcpyHostToDevice));
    owner[dev] = t;
    block[dev] = t.data_ptr<int>();
  }
  return block[dev];
}

// Set the bounded-wait limits of the current device (nanoseconds; <= 0 keeps
// the current value).  Takes effect for kernels launched afterwards.
void wait_limits_set(int64_t mbar_ns, int64_t peer_ns) {
  int* p = error_flag_ptr();
  NQ_CHECK_CUDA(cudaDeviceSynchronize());
  if (mbar_ns > 0) {
    const uint64_t v = static_cast<uint64_t>(mbar_ns);
    NQ_CHECK_CUDA(cudaMemcpy(p + 2, &v, sizeof(v), cudaMemcpyHostToDevice));
  }
  if (peer_ns > 0) {
    const uint64_t v = static_cast<uint64_t>(peer_ns);
    NQ_CHECK_CUDA(cudaMemcpy(p + 4, &v, sizeof(v), cudaMemcpyHostToDevice));
  }
}

std::vector<int64_t> wait_limits_get() {
  uint64_t lim[2];
  NQ_CHECK_CUDA(cudaMemcpy(lim, error_flag_ptr() + 2, sizeof(lim), cudaMemcpyDeviceToHost));
  return {static_cast<int64_t>(lim[0]), static_cast<int64_t>(lim[1])};
}

int64_t error_flag_read() {
  int v = 0;
  NQ_CHECK_CUDA(cudaMemcpy(&v, error_flag_ptr(), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

void error_flag_clear() { NQ_CHECK_CUDA(cudaMemset(error_flag_ptr(), 0, sizeof(int))); }

static int ew_grid(int64_t n, int threads = 256) {
  int64_t b = (n + threads - 1) / threads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(b, (int64_t)num_sms() * 16)));
}

// ------------------------------------------------------------------ SwiGLU
// gu [T, 2I] = [g | u]  ->  h [T, I] = silu(g) * u
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h,
                                  int64_t T, int I) {
  const int64_t n8 = T * I / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n8; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = v * 8;
    const int64_t t = e / I;
    const int c = static_cast<int>(e - t * I);
    float g[8], u[8], o[8];
    load8(gu + t * 2 * I + c, g);
    load8(gu + t * 2 * I + I + c, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = sigmoid_fast(g[i]);
      o[i] = g[i] * s * u[i];
    }
    store8(h + e, o);
  }
}

// dgu = [dh * u * s * (1 + g (1 - s)) | dh * g * s]
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ dgu, int64_t T, int I) {
  const int64_t n8 = T * I / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n8; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = v * 8;
    const int64_t t = e / I;
    const int c = static_cast<int>(e - t * I);
    float g[8], u[8], d[8], dg[8], du[8];
    load8(gu + t * 2 * I + c, g);
    load8(gu + t * 2 * I + I + c, u);
    load8(dh + e, d);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = sigmoid_fast(g[i]);
      dg[i] = d[i] * u[i] * s * (1.f + g[i] * (1.f - s));
      du[i] = d[i] * g[i] * s;
    }
    store8(dgu + t * 2 * I + c, dg);
    store8(dgu + t * 2 * I + I + c, du);
  }
}

torch::Tensor swiglu_fwd(torch::Tensor gu) {
  check_bf16(gu, "gu");
  TORCH_CHECK(gu.is_contiguous() && gu.size(1) % 16 == 0, "swiglu: [T, 2I] contiguous, I % 8 == 0");
  const int64_t T = gu.size(0);
  const int I = gu.size(1) / 2;
  c10::cuda::CUDAGuard g(gu.device());
  auto h = torch::empty({T, I}, gu.options());
  if (T == 0) return h;
  swiglu_fwd_kernel<<<ew_grid(T * I / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), T, I);
  NQ_CHECK_CUDA(cudaGetLastError());
  return h;
}

torch::Tensor swiglu_bwd(torch::Tensor dh, torch::Tensor gu) {
  check_bf16(dh, "dh"); check_bf16(gu, "gu");
  const int64_t T = gu.size(0);
  const int I = gu.size(1) / 2;
  c10::cuda::CUDAGuard g(gu.device());
  auto dgu = torch::empty_like(gu);
  if (T == 0) return dgu;
  auto dhc = dh.contiguous();
  swiglu_bwd_kernel<<<ew_grid(T * I / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dhc.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), T, I);
  NQ_CHECK_CUDA(cudaGetLastError());
  return dgu;
}

// -------------------------------------------------------------------- GELU
__device__ __forceinline__ float gelu_f(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }
__device__ __forceinline__ float gelu_grad(float x) {
  const float cdf = 0.5f * (1.f + erff(x * 0.70710678118654752f));
  const float pdf = 0.3989422804014327f * __expf(-0.5f * x * x);
  return cdf + x * pdf;
}

template <typename T>
__global__ void gelu_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = static_cast<T>(gelu_f(static_cast<float>(x[i])));
}
template <typename T>
__global__ void gelu_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, T* __restrict__ dx, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dx[i] = static_cast<T>(static_cast<float>(dy[i]) * gelu_grad(static_cast<float>(x[i])));
}

torch::Tensor gelu_fwd(torch::Tensor x) {
  c10::cuda::CUDAGuard g(x.device());
  auto y = torch::empty_like(x);
  const int64_t n = x.numel();
  if (n == 0) return y;
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == torch::kBFloat16)
    gelu_fwd_kernel<__nv_bfloat16><<<ew_grid(n), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), n);
  else
    gelu_fwd_kernel<float><<<ew_grid(n), 256, 0, st>>>(x.data_ptr<float>(), y.data_ptr<float>(), n);
  NQ_CHECK_CUDA(cudaGetLastError());
  return y;
}

torch::Tensor gelu_bwd(torch::Tensor dy, torch::Tensor x) {
  c10::cuda::CUDAGuard g(x.device());
  auto dx = torch::empty_like(x);
  const int64_t n = x.numel();
  if (n == 0) return dx;
  auto dyc = dy.to(x.scalar_type()).contiguous();
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == torch::kBFloat16)
    gelu_bwd_kernel<__nv_bfloat16><<<ew_grid(n), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dyc.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), n);
  else
    gelu_bwd_kernel<float><<<ew_grid(n), 256, 0, st>>>(dyc.data_ptr<float>(), x.data_ptr<float>(), dx.data_ptr<float>(), n);
  NQ_CHECK_CUDA(cudaGetLastError());
  return dx;
}

// ------------------------------------------------------- scale / axpy
template <typename T>
__global__ void scale_kernel(T* __restrict__ x, const float* __restrict__ s, int64_t n) {
  const float a = *s;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = static_cast<T>(static_cast<float>(x[i]) * a);
}

void scale_inplace(torch::Tensor x, torch::Tensor s) {
  c10::cuda::CUDAGuard g(x.device());
  auto sf = s.to(torch::kFloat32).reshape({1}).contiguous();
  const int64_t n = x.numel();
  if (n == 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == torch::kBFloat16)
    scale_kernel<__nv_bfloat16><<<ew_grid(n), 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), sf.data_ptr<float>(), n);
  else
    scale_kernel<float><<<ew_grid(n), 256, 0, st>>>(x.data_ptr<float>(), sf.data_ptr<float>(), n);
  NQ_CHECK_CUDA(cudaGetLastError());
}

__global__ void axpy_kernel(float* __restrict__ y, const float* __restrict__ x, const float* __restrict__ a, int64_t n) {
  const float s = *a;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] += s * x[i];
}

// y += a * x   (fp32, a is a device scalar)
void axpy_(torch::Tensor y, torch::Tensor x, torch::Tensor a) {
  TORCH_CHECK(y.scalar_type() == torch::kFloat32 && x.scalar_type() == torch::kFloat32, "axpy fp32");
  TORCH_CHECK(y.is_contiguous() && x.is_contiguous() && y.numel() == x.numel(), "axpy shapes");
  c10::cuda::CUDAGuard g(y.device());
  auto af = a.to(torch::kFloat32).reshape({1}).contiguous();
  const int64_t n = y.numel();
  if (n == 0) return;
  axpy_kernel<<<ew_grid(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(y.data_ptr<float>(), x.data_ptr<float>(), af.data_ptr<float>(), n);
  NQ_CHECK_CUDA(cudaGetLastError());
}

// --------------------------------------------------------------- embedding
__device__ __forceinline__ float4 load4f(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4f(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// Row gather into the fp32 residual stream from an fp32 or bf16 table.
template <typename TW>
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const TW* __restrict__ w,
                                     float* __restrict__ out, int64_t T, int H, int64_t V, int* err) {
  const int H4 = H / 4;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < T * H4; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v / H4;
    const int c = static_cast<int>(v - t * H4);
    int64_t id = ids[t];
    if (id < 0 || id >= V) { atomicCAS(err, 0, kErrBadArg); id = 0; }
    reinterpret_cast<float4*>(out)[v] = load4f(w + id * H + c * 4);
  }
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ dout,
                                     float* __restrict__ dw, int64_t T, int H, int64_t V) {
  const int H4 = H / 4;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < T * H4; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v / H4;
    const int c = static_cast<int>(v - t * H4);
    const int64_t id = ids[t];
    if (id < 0 || id >= V) continue;
    atomicAdd(reinterpret_cast<float4*>(dw + id * H) + c, reinterpret_cast<const float4*>(dout)[v]);
  }
}

torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor w) {
  const bool bf = w.scalar_type() == torch::kBFloat16;
  TORCH_CHECK((bf || w.scalar_type() == torch::kFloat32) && w.is_contiguous() && w.size(1) % 4 == 0,
              "embedding weight fp32 or bf16 [V,H%4]");
  auto idc = ids.to(torch::kInt64).contiguous();
  const int64_t T = idc.numel();
  const int H = w.size(1);
  c10::cuda::CUDAGuard g(w.device());
  auto out = torch::empty({T, H}, w.options().dtype(torch::kFloat32));
  if (T == 0) return out;
  auto st = at::cuda::getCurrentCUDAStream();
  if (bf)
    embedding_fwd_kernel<__nv_bfloat16><<<ew_grid(T * H / 4), 256, 0, st>>>(
        idc.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), out.data_ptr<float>(),
        T, H, w.size(0), error_flag_ptr());
  else
    embedding_fwd_kernel<float><<<ew_grid(T * H / 4), 256, 0, st>>>(
        idc.data_ptr<int64_t>(), w.data_ptr<float>(), out.data_ptr<float>(), T, H, w.size(0), error_flag_ptr());
  NQ_CHECK_CUDA(cudaGetLastError());
  return out;
}

void embedding_bwd(torch::Tensor ids, torch::Tensor dout, torch::Tensor dw) {
  TORCH_CHECK(dout.scalar_type() == torch::kFloat32 && dw.scalar_type() == torch::kFloat32, "embedding_bwd fp32");
  auto idc = ids.to(torch::kInt64).contiguous();
  auto dc = dout.contiguous();
  const int64_t T = idc.numel();
  const int H = dw.size(1);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(dw.device());
  embedding_bwd_kernel<<<ew_grid(T * H / 4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      idc.data_ptr<int64_t>(), dc.data_ptr<float>(), dw.data_ptr<float>(), T, H, dw.size(0));
  NQ_CHECK_CUDA(cudaGetLastError());
}

// ----------------------------------------------------------- cross-entropy
constexpr int kCEThreads = 512;
constexpr float kLog2e = 1.4426950408889634f;

// Online max/sum-exp of one row held by the block; returns (max, sumexp) in all threads.
__device__ __forceinline__ void row_lse(const __nv_bfloat16* __restrict__ x, int V, float* red_m,
                                        float* red_s, float& m_out, float& s_out) {
  float m = -INFINITY, s = 0.f;
  const int V8 = V / 8;
  for (int v = threadIdx.x; v < V8; v += blockDim.x) {
    float f[8];
    load8(x + v * 8, f);
    float lm = f[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, f[i]);
    const float nm = fmaxf(m, lm);
    float acc = s * exp2f((m - nm) * kLog2e);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += exp2f((f[i] - nm) * kLog2e);
    m = nm;
    s = acc;
  }
  for (int j = V8 * 8 + threadIdx.x; j < V; j += blockDim.x) {
    const float f = __bfloat162float(x[j]);
    const float nm = fmaxf(m, f);
    s = s * exp2f((m - nm) * kLog2e) + exp2f((f - nm) * kLog2e);
    m = nm;
  }
  // block reduce (m, s)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (nm == -INFINITY) ? 0.f : s * exp2f((m - nm) * kLog2e) + os * exp2f((om - nm) * kLog2e);
    m = nm;
  }
  __syncthreads();
  if (lane == 0) { red_m[warp] = m; red_s[warp] = s; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? red_m[lane] : -INFINITY;
    s = lane < nw ? red_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = (nm == -INFINITY) ? 0.f : s * exp2f((m - nm) * kLog2e) + os * exp2f((om - nm) * kLog2e);
      m = nm;
    }
    if (lane == 0) { red_m[0] = m; red_s[0] = s; }
  }
  __syncthreads();
  m_out = red_m[0];
  s_out = red_s[0];
}

// Per row: loss_sum += lse - x[label]; optionally x := (softmax(x) - onehot) / n_valid.
__global__ void __launch_bounds__(kCEThreads) ce_fused_kernel(
    __nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ labels, int V,
    const float* __restrict__ n_valid, float* __restrict__ loss_sum, int write_grad) {
  __shared__ float red_m[32], red_s[32];
  const int row = blockIdx.x;
  __nv_bfloat16* x = logits + static_cast<int64_t>(row) * V;
  const int64_t lab = labels[row];
  if (lab < 0 || lab >= V) {
    if (write_grad) {
      const uint4 z = make_uint4(0, 0, 0, 0);
      for (int v = threadIdx.x; v < V / 8; v += blockDim.x) reinterpret_cast<uint4*>(x)[v] = z;
      for (int j = (V / 8) * 8 + threadIdx.x; j < V; j += blockDim.x) x[j] = __float2bfloat16_rn(0.f);
    }
    return;
  }
  float m, s;
  row_lse(x, V, red_m, red_s, m, s);
  const float lse = m + __logf(s);
  const float xt = __bfloat162float(x[lab]);
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(loss_sum, lse - xt);
  if (!write_grad) return;
  const float inv = 1.f / fmaxf(*n_valid, 1.f);
  for (int v = threadIdx.x; v < V / 8; v += blockDim.x) {
    float f[8];
    load8(x + v * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = v * 8 + i;
      f[i] = (exp2f((f[i] - lse) * kLog2e) - (j == lab ? 1.f : 0.f)) * inv;
    }
    store8(x + v * 8, f);
  }
  for (int j = (V / 8) * 8 + threadIdx.x; j < V; j += blockDim.x) {
    const float f = __bfloat162float(x[j]);
    x[j] = __float2bfloat16_rn((exp2f((f - lse) * kLog2e) - (j == lab ? 1.f : 0.f)) * inv);
  }
}

__global__ void __launch_bounds__(kCEThreads) ce_lse_kernel(
    const __nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ labels, int V,
    float* __restrict__ lse_out, float* __restrict__ tgt_out) {
  __shared__ float red_m[32], red_s[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + static_cast<int64_t>(row) * V;
  float m, s;
  row_lse(x, V, red_m, red_s, m, s);
  if (threadIdx.x == 0) {
    const int64_t lab = labels[row];
    lse_out[row] = m + __logf(s);
    tgt_out[row] = (lab >= 0 && lab < V) ? __bfloat162float(x[lab]) : 0.f;
  }
}

// x := (softmax(x) - onehot) * g[row]   (g = 0 for ignored rows)
__global__ void __launch_bounds__(kCEThreads) ce_grad_kernel(
    __nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ labels, int V,
    const float* __restrict__ lse, const float* __restrict__ gscale) {
  const int row = blockIdx.x;
  __nv_bfloat16* x = logits + static_cast<int64_t>(row) * V;
  const int64_t lab = labels[row];
  const bool valid = lab >= 0 && lab < V;
  const float g = valid ? gscale[row] : 0.f;  // dL/d(row loss)
  const float l = lse[row];
  for (int v = threadIdx.x; v < V / 8; v += blockDim.x) {
    float f[8];
    load8(x + v * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = v * 8 + i;
      f[i] = (exp2f((f[i] - l) * kLog2e) - (j == lab ? 1.f : 0.f)) * g;
    }
    store8(x + v * 8, f);
  }
  for (int j = (V / 8) * 8 + threadIdx.x; j < V; j += blockDim.x) {
    const float f = __bfloat162float(x[j]);
    x[j] = __float2bfloat16_rn((exp2f((f - l) * kLog2e) - (j == lab ? 1.f : 0.f)) * g);
  }
}

__global__ void count_valid_kernel(const int64_t* __restrict__ labels, int64_t n, float* out) {
  __shared__ float red[32];
  float c = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    c += labels[i] != -100 ? 1.f : 0.f;
  c = block_sum(c, red);
  if (threadIdx.x == 0) atomicAdd(out, c);
}

torch::Tensor ce_count_valid(torch::Tensor labels) {
  auto lc = labels.to(torch::kInt64).contiguous();
  c10::cuda::CUDAGuard g(labels.device());
  auto out = torch::zeros({}, labels.options().dtype(torch::kFloat32));
  const int64_t n = lc.numel();
  if (n) count_valid_kernel<<<std::min<int64_t>(64, (n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(lc.data_ptr<int64_t>(), n, out.data_ptr<float>());
  NQ_CHECK_CUDA(cudaGetLastError());
  return out;
}

void ce_fused_chunk(torch::Tensor logits, torch::Tensor labels, torch::Tensor n_valid, torch::Tensor loss_sum, bool write_grad) {
  check_bf16(logits, "logits");
  TORCH_CHECK(logits.is_contiguous() && logits.size(1) % 8 == 0, "ce: logits contiguous, V % 8 == 0");
  auto lc = labels.to(torch::kInt64).contiguous();
  const int R = logits.size(0), V = logits.size(1);
  if (R == 0) return;
  c10::cuda::CUDAGuard g(logits.device());
  ce_fused_kernel<<<R, kCEThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), lc.data_ptr<int64_t>(), V,
      n_valid.data_ptr<float>(), loss_sum.data_ptr<float>(), write_grad ? 1 : 0);
  NQ_CHECK_CUDA(cudaGetLastError());
}

void ce_lse_chunk(torch::Tensor logits, torch::Tensor labels, torch::Tensor lse, torch::Tensor tgt) {
  check_bf16(logits, "logits");
  auto lc = labels.to(torch::kInt64).contiguous();
  const int R = logits.size(0), V = logits.size(1);
  if (R == 0) return;
  c10::cuda::CUDAGuard g(logits.device());
  ce_lse_kernel<<<R, kCEThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), lc.data_ptr<int64_t>(), V,
      lse.data_ptr<float>(), tgt.data_ptr<float>());
  NQ_CHECK_CUDA(cudaGetLastError());
}

// g is dL/d(loss_row); writes d(loss_row)/d(logits) * g
void ce_grad_chunk(torch::Tensor logits, torch::Tensor labels, torch::Tensor lse, torch::Tensor g_in) {
  check_bf16(logits, "logits");
  auto lc = labels.to(torch::kInt64).contiguous();
  auto gneg = g_in.to(torch::kFloat32).contiguous();
  const int R = logits.size(0), V = logits.size(1);
  if (R == 0) return;
  c10::cuda::CUDAGuard g(logits.device());
  ce_grad_kernel<<<R, kCEThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), lc.data_ptr<int64_t>(), V,
      lse.data_ptr<float>(), gneg.data_ptr<float>());
  NQ_CHECK_CUDA(cudaGetLastError());
}

// ------------------------------------------------------ grad norm + AdamW
__global__ void sum_squares_kernel(const float* __restrict__ x, int64_t n, float* out) {
  __shared__ float red[32];
  float s = 0.f;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    s += x[i] * x[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) atomicAdd(out, s);
}

torch::Tensor sum_squares(torch::Tensor x) {
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous(), "sum_squares fp32 contiguous");
  c10::cuda::CUDAGuard g(x.device());
  auto out = torch::zeros({}, x.options());
  const int64_t n = x.numel();
  if (n) sum_squares_kernel<<<ew_grid(n / 4 + 1, 512), 512, 0, at::cuda::getCurrentCUDAStream()>>>(x.data_ptr<float>(), n, out.data_ptr<float>());
  NQ_CHECK_CUDA(cudaGetLastError());
  return out;
}

template <bool WRITE_BF16>
__global__ void adamw_flat_kernel(float* __restrict__ p, const float* __restrict__ g,
                                  float* __restrict__ m, float* __restrict__ v,
                                  __nv_bfloat16* __restrict__ comp, const float* __restrict__ clip,
                                  int64_t begin, int64_t end, int64_t sbase, int64_t decay_end,
                                  float lr_d, float lr_n, float b1, float b2, float eps, float wd,
                                  float bc1, float bc2) {
  // m / v hold the optimizer state of flat elements [sbase, sbase + numel):
  // the whole store (sbase 0) or only this rank's shard (sbase = begin).
  m -= sbase;
  v -= sbase;
  const float cs = *clip;
  const float rbc1 = 1.f / bc1, rbc2 = 1.f / bc2;
  const int64_t n4 = (end - begin) / 4;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n4; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = begin + q * 4;
    const bool decay = i < decay_end;
    const float lr = decay ? lr_d : lr_n;
    const float w = decay ? wd : 0.f;
    float4 pv = *reinterpret_cast<float4*>(p + i);
    const float4 gv = *reinterpret_cast<const float4*>(g + i);
    float4 mv = *reinterpret_cast<float4*>(m + i);
    float4 vv = *reinterpret_cast<float4*>(v + i);
    float* pp = &pv.x; const float* gg = &gv.x; float* mm = &mv.x; float* vq = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gr = gg[k] * cs;
      float x = pp[k] * (1.f - lr * w);
      mm[k] = b1 * mm[k] + (1.f - b1) * gr;
      vq[k] = b2 * vq[k] + (1.f - b2) * gr * gr;
      const float denom = sqrtf(vq[k] * rbc2) + eps;
      pp[k] = x - lr * (mm[k] * rbc1) / denom;
    }
    *reinterpret_cast<float4*>(p + i) = pv;
    *reinterpret_cast<float4*>(m + i) = mv;
    *reinterpret_cast<float4*>(v + i) = vv;
    if (WRITE_BF16) {
      __nv_bfloat162 a = __floats2bfloat162_rn(pv.x, pv.y), b = __floats2bfloat162_rn(pv.z, pv.w);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&a);
      u.y = *reinterpret_cast<uint32_t*>(&b);
      *reinterpret_cast<uint2*>(comp + i) = u;
    }
  }
}

void adamw_flat(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v,
                torch::Tensor comp, torch::Tensor clip, int64_t begin, int64_t end, int64_t sbase,
                int64_t decay_end, double lr_d, double lr_n, double b1, double b2, double eps,
                double wd, double bc1, double bc2) {
  TORCH_CHECK(begin % 4 == 0 && end % 4 == 0 && sbase % 4 == 0, "adamw range must be 4-aligned");
  TORCH_CHECK(sbase <= begin && end - sbase <= m.numel() && m.numel() == v.numel(),
              "adamw: optimizer state does not cover the updated range");
  c10::cuda::CUDAGuard gd(p.device());
  const int64_t n = end - begin;
  if (n <= 0) return;
  auto st = at::cuda::getCurrentCUDAStream();
  auto cl = clip.to(torch::kFloat32).reshape({1}).contiguous();
  if (comp.numel() > 0) {
    adamw_flat_kernel<true><<<ew_grid(n / 4, 256), 256, 0, st>>>(
        p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(comp.data_ptr()), cl.data_ptr<float>(), begin, end, sbase, decay_end,
        (float)lr_d, (float)lr_n, (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2);
  } else {
    adamw_flat_kernel<false><<<ew_grid(n / 4, 256), 256, 0, st>>>(
        p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), nullptr,
        cl.data_ptr<float>(), begin, end, sbase, decay_end, (float)lr_d, (float)lr_n, (float)b1, (float)b2,
        (float)eps, (float)wd, (float)bc1, (float)bc2);
  }
  NQ_CHECK_CUDA(cudaGetLastError());
}

}  // namespace nq
