// Fused per-head QK-RMSNorm + NeoX RoPE on the packed q|k|v projection.
//
// Forward: one warp per (token, head) of q and k; each lane owns PPL rotation
// pairs (i, i + D/2).  Reads the bf16 GEMM output, writes bf16 q|k rows
// [T, (Hq+Hk)*D] and fp32 1/rms per (token, head).  Matches the reference's
// numerics: normalise in fp32, round to the activation dtype, scale by the
// weight, rotate in fp32, round once (reference: model/attention.py:88-95,
// model/norm.py:20-22, model/rope.py:146-161).
// Backward: inverse rotation, RMSNorm backward, weight gradients reduced per
// warp in registers and flushed once per warp.
#include "common.cuh"
#include "tmap.h"

namespace nq {

template <int PPL, typename TG>
__global__ void __launch_bounds__(256) qknorm_rope_fwd_kernel(
    const __nv_bfloat16* __restrict__ qkv, const float* __restrict__ qw,
    const float* __restrict__ kw, const float* __restrict__ cosT, const float* __restrict__ sinT,
    const int64_t* __restrict__ pos, __nv_bfloat16* __restrict__ out, float* __restrict__ rstd,
    int T, int S, int Hq, int Hk, int D, float eps) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int Hqk = Hq + Hk;
  const int W = (Hq + 2 * Hk) * D;
  const int half = D / 2;
  const int64_t items = static_cast<int64_t>(T) * Hqk;
  for (int64_t it = gw; it < items; it += warps) {
    const int t = static_cast<int>(it / Hqk);
    const int h = static_cast<int>(it - static_cast<int64_t>(t) * Hqk);
    const bool is_q = h < Hq;
    const float* w = is_q ? qw : kw;
    const __nv_bfloat16* src = qkv + static_cast<int64_t>(t) * W + h * D;
    float x1[PPL], x2[PPL];
    float ss = 0.f;
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      const int i = lane * PPL + p;
      x1[p] = __bfloat162float(src[i]);
      x2[p] = __bfloat162float(src[i + half]);
      ss += x1[p] * x1[p] + x2[p] * x2[p];
    }
    float r = 1.f;
    if (w != nullptr) {
      ss = warp_sum(ss);
      r = rsqrtf(ss / D + eps);
#pragma unroll
      for (int p = 0; p < PPL; ++p) {
        const int i = lane * PPL + p;
        x1[p] = bf16r(x1[p] * r) * w[i];
        x2[p] = bf16r(x2[p] * r) * w[i + half];
      }
    }
    if (lane == 0) rstd[it] = r;
    const int s = t % S;
    const int64_t ps = (pos != nullptr) ? pos[t] : s;
    __nv_bfloat16* dst = out + static_cast<int64_t>(t) * Hqk * D + h * D;
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      const int i = lane * PPL + p;
      const float c = cosT[ps * half + i], sn = sinT[ps * half + i];
      dst[i] = __float2bfloat16_rn(x1[p] * c - x2[p] * sn);
      dst[i + half] = __float2bfloat16_rn(x2[p] * c + x1[p] * sn);
    }
  }
}

template <int PPL, typename TG>
__global__ void __launch_bounds__(256) qknorm_rope_bwd_kernel(
    const TG* __restrict__ dqk, const __nv_bfloat16* __restrict__ qkv,
    const float* __restrict__ qw, const float* __restrict__ kw, const float* __restrict__ rstd,
    const float* __restrict__ cosT, const float* __restrict__ sinT,
    const int64_t* __restrict__ pos, __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dqw,
    float* __restrict__ dkw, int T, int S, int Hq, int Hk, int D) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int Hqk = Hq + Hk;
  const int W = (Hq + 2 * Hk) * D;
  const int half = D / 2;
  float aq1[PPL], aq2[PPL], ak1[PPL], ak2[PPL];
#pragma unroll
  for (int p = 0; p < PPL; ++p) { aq1[p] = aq2[p] = ak1[p] = ak2[p] = 0.f; }
  const int64_t items = static_cast<int64_t>(T) * Hqk;
  for (int64_t it = gw; it < items; it += warps) {
    const int t = static_cast<int>(it / Hqk);
    const int h = static_cast<int>(it - static_cast<int64_t>(t) * Hqk);
    const bool is_q = h < Hq;
    const float* w = is_q ? qw : kw;
    const int s = t % S;
    const int64_t ps = (pos != nullptr) ? pos[t] : s;
    const TG* g = dqk + static_cast<int64_t>(t) * Hqk * D + h * D;
    float dn1[PPL], dn2[PPL];
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      const int i = lane * PPL + p;
      const float c = cosT[ps * half + i], sn = sinT[ps * half + i];
      const float g1 = static_cast<float>(g[i]), g2 = static_cast<float>(g[i + half]);
      dn1[p] = g1 * c + g2 * sn;
      dn2[p] = -g1 * sn + g2 * c;
    }
    __nv_bfloat16* dst = dqkv + static_cast<int64_t>(t) * W + h * D;
    if (w == nullptr) {
#pragma unroll
      for (int p = 0; p < PPL; ++p) {
        const int i = lane * PPL + p;
        dst[i] = __float2bfloat16_rn(dn1[p]);
        dst[i + half] = __float2bfloat16_rn(dn2[p]);
      }
      continue;
    }
    const float r = rstd[it];
    const __nv_bfloat16* src = qkv + static_cast<int64_t>(t) * W + h * D;
    float xh1[PPL], xh2[PPL], du1[PPL], du2[PPL];
    float dot = 0.f;
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      const int i = lane * PPL + p;
      xh1[p] = __bfloat162float(src[i]) * r;
      xh2[p] = __bfloat162float(src[i + half]) * r;
      const float u1 = bf16r(xh1[p]), u2 = bf16r(xh2[p]);
      du1[p] = dn1[p] * w[i];
      du2[p] = dn2[p] * w[i + half];
      if (is_q) { aq1[p] += dn1[p] * u1; aq2[p] += dn2[p] * u2; }
      else { ak1[p] += dn1[p] * u1; ak2[p] += dn2[p] * u2; }
      dot += du1[p] * xh1[p] + du2[p] * xh2[p];
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      const int i = lane * PPL + p;
      dst[i] = __float2bfloat16_rn(r * (du1[p] - xh1[p] * dot));
      dst[i + half] = __float2bfloat16_rn(r * (du2[p] - xh2[p] * dot));
    }
  }
  if (dqw != nullptr && dkw != nullptr) {
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      const int i = lane * PPL + p;
      atomicAdd(dqw + i, aq1[p]);
      atomicAdd(dqw + i + half, aq2[p]);
      atomicAdd(dkw + i, ak1[p]);
      atomicAdd(dkw + i + half, ak2[p]);
    }
  }
}


static int rope_grid(int64_t items) {
  int64_t blocks = (items + 7) / 8;  // 8 warps per block
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, num_sms() * 8)));
}

#define NQ_PPL_DISPATCH(D, ...)                                        \
  switch (D) {                                                         \
    case 64: { constexpr int PPL = 1; __VA_ARGS__; break; }            \
    case 128: { constexpr int PPL = 2; __VA_ARGS__; break; }           \
    case 256: { constexpr int PPL = 4; __VA_ARGS__; break; }           \
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
  NQ_PPL_DISPATCH(D, qknorm_rope_fwd_kernel<PPL, float><<<rope_grid((int64_t)T * (Hq + Hk)), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), opt_f32(qw), opt_f32(kw),
      cc.data_ptr<float>(), sc.data_ptr<float>(), pp,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rstd.data_ptr<float>(), T, S, Hq, Hk, D,
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
    NQ_PPL_DISPATCH(D, qknorm_rope_bwd_kernel<PPL, float><<<rope_grid((int64_t)T * (Hq + Hk)), 256, 0, st>>>(
        dqkc.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
        opt_f32(qw), opt_f32(kw), rstd.data_ptr<float>(), cc.data_ptr<float>(), sc.data_ptr<float>(),
        pp, reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), dq, dk, T, S, Hq, Hk, D));
  } else {
    NQ_PPL_DISPATCH(D, qknorm_rope_bwd_kernel<PPL, __nv_bfloat16><<<rope_grid((int64_t)T * (Hq + Hk)), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(dqkc.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
        opt_f32(qw), opt_f32(kw), rstd.data_ptr<float>(), cc.data_ptr<float>(), sc.data_ptr<float>(),
        pp, reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), dq, dk, T, S, Hq, Hk, D));
  }
  NQ_CHECK_CUDA(cudaGetLastError());
}

}  // namespace nq
