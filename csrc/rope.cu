// Fused per-head QK-RMSNorm + NeoX RoPE on the packed q|k|v projection.
//
// One warp per token (all of its heads); lane l owns the EPL = D/32 contiguous elements
// [l*EPL, (l+1)*EPL) so every access is a 4-16 byte vector.  Lanes 0-15 hold
// the first half of the head, lanes 16-31 the second; the rotation partner of
// element i is element i + D/2, i.e. the same slot of lane l^16, exchanged with
// one shuffle.  Forward writes bf16 q|k rows [T, (Hq+Hk)*D] and fp32 1/rms per
// (token, head).  Numerics follow the reference: normalise in fp32, round to
// the activation dtype, scale by the weight, rotate in fp32, round once
// (reference: model/attention.py:88-95, model/norm.py:20-22,
// model/rope.py:146-161).  Backward: inverse rotation, RMSNorm backward,
// weight gradients reduced per warp in registers and flushed once per warp.
#include "common.cuh"
#include "tmap.h"

namespace nq {

template <int EPL>
__device__ __forceinline__ void ld_bf16(const __nv_bfloat16* p, float (&v)[EPL]) {
  if constexpr (EPL == 2) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    v[0] = f.x; v[1] = f.y;
  } else if constexpr (EPL == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else {
    load8(p, v);
  }
}

template <int EPL>
__device__ __forceinline__ void st_bf16(__nv_bfloat16* p, const float (&v)[EPL]) {
  if constexpr (EPL == 2) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v[0], v[1]);
  } else if constexpr (EPL == 4) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
  } else {
    store8(p, v);
  }
}

template <int EPL>
__device__ __forceinline__ void ld_f32(const float* p, float (&v)[EPL]) {
#pragma unroll
  for (int i = 0; i < EPL; i += 2) {
    const float2 f = *reinterpret_cast<const float2*>(p + i);
    v[i] = f.x; v[i + 1] = f.y;
  }
}

template <int EPL>
__device__ __forceinline__ void ld_grad(const float* p, float (&v)[EPL]) { ld_f32<EPL>(p, v); }
template <int EPL>
__device__ __forceinline__ void ld_grad(const __nv_bfloat16* p, float (&v)[EPL]) { ld_bf16<EPL>(p, v); }

// Heads processed per inner step: their loads are issued together so each warp
// keeps several independent row reads in flight.
constexpr int kRopeUnroll = 4;
constexpr int kRopeBwdUnroll = 2;  // the backward holds three rows per head in registers

template <int D>
__global__ void __launch_bounds__(256) qknorm_rope_fwd_kernel(
    const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ qw,
    const float* __restrict__ kw, const float* __restrict__ cosT, const float* __restrict__ sinT,
    const int64_t* __restrict__ pos, __nv_bfloat16* __restrict__ out, float* __restrict__ rstd,
    int T, int S, int Hq, int Hk, float eps) {
  constexpr int EPL = D / 32;
  constexpr int half = D / 2;
  const int lane = threadIdx.x & 31;
  const bool hi = lane >= 16;
  const int e0 = lane * EPL;           // first element of this lane
  const int f0 = e0 & (half - 1);      // frequency index of the first element
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int Hqk = Hq + Hk;
  const int W = (Hq + 2 * Hk) * D;
  float wq[EPL], wk[EPL];
  if (qw != nullptr) { ld_f32<EPL>(qw + e0, wq); ld_f32<EPL>(kw + e0, wk); }
  // one warp per token: the cos/sin row is read once for all of its heads
  for (int t = gw; t < T; t += warps) {
    const int64_t ps = (pos != nullptr) ? pos[t] : (t % S);
    float c[EPL], sn[EPL];
    ld_f32<EPL>(cosT + ps * half + f0, c);
    ld_f32<EPL>(sinT + ps * half + f0, sn);
    const __nv_bfloat16* src = qkv + static_cast<int64_t>(t) * W + e0;
    __nv_bfloat16* dst = out + static_cast<int64_t>(t) * Hqk * D + e0;
    for (int h0 = 0; h0 < Hqk; h0 += kRopeUnroll) {
      float x[kRopeUnroll][EPL];
#pragma unroll
      for (int u = 0; u < kRopeUnroll; ++u)
        if (h0 + u < Hqk) ld_bf16<EPL>(src + (h0 + u) * D, x[u]);
#pragma unroll
      for (int u = 0; u < kRopeUnroll; ++u) {
        const int h = h0 + u;
        if (h >= Hqk) break;
        float r = 1.f;
        if (qw != nullptr) {
          float ss = 0.f;
#pragma unroll
          for (int i = 0; i < EPL; ++i) ss += x[u][i] * x[u][i];
          r = rsqrtf(warp_sum(ss) / D + eps);
          const bool is_q = h < Hq;
#pragma unroll
          for (int i = 0; i < EPL; ++i) x[u][i] = bf16r(x[u][i] * r) * (is_q ? wq[i] : wk[i]);
        }
        if (lane == 0) rstd[static_cast<int64_t>(t) * Hqk + h] = r;
        float o[EPL];
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float pr = __shfl_xor_sync(0xffffffffu, x[u][i], 16);
          // first half: x1*c - x2*s ; second half: x2*c + x1*s (the partner is the other half)
          o[i] = hi ? fmaf(x[u][i], c[i], pr * sn[i]) : fmaf(x[u][i], c[i], -pr * sn[i]);
        }
        st_bf16<EPL>(dst + h * D, o);
      }
    }
  }
}

template <int D, typename TG>
__global__ void __launch_bounds__(256, (D <= 128 ? 3 : 1)) qknorm_rope_bwd_kernel(
    const TG* __restrict__ dqk, const __nv_bfloat16* __restrict__ qkv,
    const float* __restrict__ qw, const float* __restrict__ kw, const float* __restrict__ rstd,
    const float* __restrict__ cosT, const float* __restrict__ sinT,
    const int64_t* __restrict__ pos, __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dqw,
    float* __restrict__ dkw, int T, int S, int Hq, int Hk) {
  constexpr int EPL = D / 32;
  constexpr int half = D / 2;
  const int lane = threadIdx.x & 31;
  const bool hi = lane >= 16;
  const int e0 = lane * EPL;
  const int f0 = e0 & (half - 1);
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int Hqk = Hq + Hk;
  const int W = (Hq + 2 * Hk) * D;
  const bool norm = qw != nullptr;
  float wq[EPL], wk[EPL], aq[EPL], ak[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) { aq[i] = 0.f; ak[i] = 0.f; wq[i] = 1.f; wk[i] = 1.f; }
  if (norm) { ld_f32<EPL>(qw + e0, wq); ld_f32<EPL>(kw + e0, wk); }
  for (int t = gw; t < T; t += warps) {
    const int64_t ps = (pos != nullptr) ? pos[t] : (t % S);
    float c[EPL], sn[EPL];
    ld_f32<EPL>(cosT + ps * half + f0, c);
    ld_f32<EPL>(sinT + ps * half + f0, sn);
    const TG* gsrc = dqk + static_cast<int64_t>(t) * Hqk * D + e0;
    const __nv_bfloat16* xsrc = qkv + static_cast<int64_t>(t) * W + e0;
    __nv_bfloat16* dst = dqkv + static_cast<int64_t>(t) * W + e0;
    for (int h0 = 0; h0 < Hqk; h0 += kRopeBwdUnroll) {
      float g[kRopeBwdUnroll][EPL], x[kRopeBwdUnroll][EPL], rr[kRopeBwdUnroll];
#pragma unroll
      for (int u = 0; u < kRopeBwdUnroll; ++u) {
        if (h0 + u < Hqk) {
          ld_grad<EPL>(gsrc + (h0 + u) * D, g[u]);
          if (norm) {
            ld_bf16<EPL>(xsrc + (h0 + u) * D, x[u]);
            rr[u] = rstd[static_cast<int64_t>(t) * Hqk + h0 + u];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kRopeBwdUnroll; ++u) {
        const int h = h0 + u;
        if (h >= Hqk) break;
        float dn[EPL];
        // inverse rotation: first half g1*c + g2*s ; second half g2*c - g1*s
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float pr = __shfl_xor_sync(0xffffffffu, g[u][i], 16);
          dn[i] = hi ? fmaf(g[u][i], c[i], -pr * sn[i]) : fmaf(g[u][i], c[i], pr * sn[i]);
        }
        if (!norm) {
          st_bf16<EPL>(dst + h * D, dn);
          continue;
        }
        const bool is_q = h < Hq;
        const float r = rr[u];
        float du[EPL], o[EPL];
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float xh = x[u][i] * r;
          const float uu = bf16r(xh);
          du[i] = dn[i] * (is_q ? wq[i] : wk[i]);
          if (is_q) aq[i] += dn[i] * uu; else ak[i] += dn[i] * uu;
          dot += du[i] * xh;
          x[u][i] = xh;
        }
        dot = warp_sum(dot) / D;
#pragma unroll
        for (int i = 0; i < EPL; ++i) o[i] = r * (du[i] - x[u][i] * dot);
        st_bf16<EPL>(dst + h * D, o);
      }
    }
  }
  if (dqw == nullptr || dkw == nullptr) return;
  // Block-level reduction of the weight gradients in shared memory, then one
  // global atomic per element per block.
  __shared__ float red[2 * D];
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) red[i] = 0.f;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    atomicAdd(&red[e0 + i], aq[i]);
    atomicAdd(&red[D + e0 + i], ak[i]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) {
    const float v = red[i];
    if (v != 0.f) atomicAdd(i < D ? dqw + i : dkw + (i - D), v);
  }
}

static int rope_grid(int64_t tokens, int per_sm = 8) {
  int64_t blocks = (tokens + 7) / 8;  // 8 warps per block, one token per warp
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, num_sms() * per_sm)));
}

#define NQ_D_DISPATCH(D, ...)                                          \
  switch (D) {                                                         \
    case 64: { constexpr int DD = 64; __VA_ARGS__; break; }            \
    case 128: { constexpr int DD = 128; __VA_ARGS__; break; }          \
    case 256: { constexpr int DD = 256; __VA_ARGS__; break; }          \
    default: TORCH_CHECK(false, "head_dim must be 64, 128 or 256");    \
  }

static float* opt_f32(const c10::optional<torch::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr<float>() : nullptr;
}

std::vector<torch::Tensor> qknorm_rope_fwd(torch::Tensor qkv, c10::optional<torch::Tensor> qw,
                                           c10::optional<torch::Tensor> kw, torch::Tensor cosT,
                                           torch::Tensor sinT, c10::optional<torch::Tensor> pos,
                                           int64_t B, int64_t S, int64_t Hq, int64_t Hk, int64_t D,
                                           double eps) {
  check_bf16(qkv, "qkv");
  TORCH_CHECK(qkv.is_contiguous() && qkv.size(1) == (Hq + 2 * Hk) * D, "qkv shape");
  const int T = qkv.size(0);
  c10::cuda::CUDAGuard g(qkv.device());
  auto out = torch::empty({T, (Hq + Hk) * D}, qkv.options());
  auto rstd = torch::empty({T, Hq + Hk}, qkv.options().dtype(torch::kFloat32));
  if (T == 0) return {out, rstd};
  torch::Tensor posc;
  const int64_t* pp = nullptr;
  if (pos.has_value() && pos->defined()) {
    posc = pos->to(torch::kInt64).contiguous();
    pp = posc.data_ptr<int64_t>();
  }
  auto cc = cosT.contiguous(), sc = sinT.contiguous();
  auto st = at::cuda::getCurrentCUDAStream();
  NQ_D_DISPATCH(D, qknorm_rope_fwd_kernel<DD><<<rope_grid(T), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), opt_f32(qw), opt_f32(kw),
      cc.data_ptr<float>(), sc.data_ptr<float>(), pp,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rstd.data_ptr<float>(), T, S, Hq, Hk,
      (float)eps));
  NQ_CHECK_CUDA(cudaGetLastError());
  return {out, rstd};
}

void qknorm_rope_bwd(torch::Tensor dqk, torch::Tensor qkv, c10::optional<torch::Tensor> qw,
                     c10::optional<torch::Tensor> kw, torch::Tensor rstd, torch::Tensor cosT,
                     torch::Tensor sinT, c10::optional<torch::Tensor> pos, torch::Tensor dqkv,
                     c10::optional<torch::Tensor> dqw, c10::optional<torch::Tensor> dkw,
                     int64_t B, int64_t S, int64_t Hq, int64_t Hk, int64_t D) {
  const int T = qkv.size(0);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(qkv.device());
  torch::Tensor posc;
  const int64_t* pp = nullptr;
  if (pos.has_value() && pos->defined()) {
    posc = pos->to(torch::kInt64).contiguous();
    pp = posc.data_ptr<int64_t>();
  }
  auto cc = cosT.contiguous(), sc = sinT.contiguous();
  // Weight-gradient scratch when only one of q/k needs it.
  torch::Tensor zq, zk;
  float* dq = opt_f32(dqw);
  float* dk = opt_f32(dkw);
  if (opt_f32(qw) != nullptr && (dq == nullptr || dk == nullptr)) {
    if (dq == nullptr) { zq = torch::zeros({D}, qkv.options().dtype(torch::kFloat32)); dq = zq.data_ptr<float>(); }
    if (dk == nullptr) { zk = torch::zeros({D}, qkv.options().dtype(torch::kFloat32)); dk = zk.data_ptr<float>(); }
  }
  auto st = at::cuda::getCurrentCUDAStream();
  auto dqkc = dqk.contiguous();
  if (dqkc.scalar_type() == torch::kFloat32) {
    NQ_D_DISPATCH(D, qknorm_rope_bwd_kernel<DD, float><<<rope_grid(T, 3), 256, 0, st>>>(
        dqkc.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
        opt_f32(qw), opt_f32(kw), rstd.data_ptr<float>(), cc.data_ptr<float>(), sc.data_ptr<float>(),
        pp, reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), dq, dk, T, S, Hq, Hk));
  } else {
    NQ_D_DISPATCH(D, qknorm_rope_bwd_kernel<DD, __nv_bfloat16><<<rope_grid(T, 3), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(dqkc.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
        opt_f32(qw), opt_f32(kw), rstd.data_ptr<float>(), cc.data_ptr<float>(), sc.data_ptr<float>(),
        pp, reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), dq, dk, T, S, Hq, Hk));
  }
  NQ_CHECK_CUDA(cudaGetLastError());
}

}  // namespace nq
