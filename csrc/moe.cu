// Mixture-of-experts routing kernels: router softmax/top-k/renorm with aux
// statistics, the stable counting-sort dispatch plan, row gather, weighted
// combine and their backward passes.  No host synchronisation: every size the
// grouped GEMMs need lives in device memory (offsets), and the permuted buffer
// has the static capacity N*k + E*pad.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace nq {

constexpr int kMaxE = 256;
constexpr int kMaxK = 16;

// ------------------------------------------------------------------ router
template <typename TL>
__global__ void router_fwd_kernel(const TL* __restrict__ logits, int N, int E, int K, int norm,
                                  float* __restrict__ w_out, int* __restrict__ idx_out,
                                  float* __restrict__ counts, float* __restrict__ psum, int* err) {
  __shared__ float s_cnt[kMaxE], s_psum[kMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) { s_cnt[e] = 0.f; s_psum[e] = 0.f; }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  constexpr int PER = kMaxE / 32;
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < N; t += warps) {
    float p[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      p[i] = (e < E) ? static_cast<float>(logits[static_cast<int64_t>(t) * E + e]) : -INFINITY;
      mx = fmaxf(mx, p[i]);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      p[i] = (lane + 32 * i < E) ? __expf(p[i] - mx) : 0.f;
      sum += p[i];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
    // A non-finite logit makes the row's probabilities NaN; the top-k below
    // must still pick K distinct experts in [0, E), so such a row routes on
    // zero probabilities (lowest expert ids) and the error word records it.
    bool bad = false;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      p[i] *= inv;
      if (!(p[i] >= 0.f)) {  // NaN
        bad |= (lane + 32 * i < E);
        p[i] = 0.f;
      }
      if (lane + 32 * i < E) atomicAdd(&s_psum[lane + 32 * i], p[i]);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicCAS(err, 0, kErrBadArg);
    // top-k by repeated warp argmax (ties -> lower expert id)
    float selv[kMaxK];
    int seli[kMaxK];
    bool taken[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) taken[i] = false;
    float selsum = 0.f;
    for (int j = 0; j < K; ++j) {
      float bv = -1.f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !taken[i] && (p[i] > bv || (p[i] == bv && e < bi))) { bv = p[i]; bi = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (bi >= E) {  // cannot happen with finite probabilities and K <= E
        if (lane == 0) atomicCAS(err, 0, kErrBadArg);
        bi = 0;
        bv = 0.f;
      }
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (lane + 32 * i == bi) taken[i] = true;
      selv[j] = bv;
      seli[j] = bi;
      selsum += bv;
    }
    if (lane == 0) {
      const float rn = norm && selsum > 0.f ? 1.f / selsum : 1.f;
      for (int j = 0; j < K; ++j) {
        w_out[static_cast<int64_t>(t) * K + j] = selv[j] * rn;
        idx_out[static_cast<int64_t>(t) * K + j] = seli[j];
        atomicAdd(&s_cnt[seli[j]], 1.f);
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    if (s_cnt[e] != 0.f) atomicAdd(&counts[e], s_cnt[e]);
    if (s_psum[e] != 0.f) atomicAdd(&psum[e], s_psum[e]);
  }
}

template <typename TL>
__global__ void router_bwd_kernel(const TL* __restrict__ logits, const float* __restrict__ w,
                                  const int* __restrict__ idx, const float* __restrict__ dw,
                                  const float* __restrict__ dpsum, int N, int E, int K, int norm,
                                  TL* __restrict__ dlogits) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  constexpr int PER = kMaxE / 32;
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < N; t += warps) {
    float p[PER], dp[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      p[i] = (e < E) ? static_cast<float>(logits[static_cast<int64_t>(t) * E + e]) : -INFINITY;
      mx = fmaxf(mx, p[i]);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      p[i] = (lane + 32 * i < E) ? __expf(p[i] - mx) : 0.f;
      sum += p[i];
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      p[i] /= sum;
      dp[i] = (lane + 32 * i < E) ? dpsum[lane + 32 * i] : 0.f;
    }
    // contributions of the selected weights
    float selsum = 0.f, wdw = 0.f;
    for (int j = 0; j < K; ++j) {
      const int e = idx[static_cast<int64_t>(t) * K + j];
      const float pe = __shfl_sync(0xffffffffu, p[(e >> 5) % PER], e & 31);
      selsum += pe;
      wdw += w[static_cast<int64_t>(t) * K + j] * dw[static_cast<int64_t>(t) * K + j];
    }
    for (int j = 0; j < K; ++j) {
      const int e = idx[static_cast<int64_t>(t) * K + j];
      const float g = dw[static_cast<int64_t>(t) * K + j];
      const float add = norm ? (g - wdw) / selsum : g;
      if ((e & 31) == lane) dp[e >> 5] += add;
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) dot += p[i] * dp[i];
    dot = warp_sum(dot);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < E) dlogits[static_cast<int64_t>(t) * E + e] = static_cast<TL>(p[i] * (dp[i] - dot));
    }
  }
}

static int warp_grid(int64_t items) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((items + 7) / 8, num_sms() * 8)));
}

std::vector<torch::Tensor> router_fwd(torch::Tensor logits, int64_t K, bool norm) {
  TORCH_CHECK(logits.is_contiguous() && logits.dim() == 2, "router: logits [N,E] contiguous");
  const int N = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E <= kMaxE && K <= kMaxK && K <= E, "router: E <= 256, k <= 16");
  c10::cuda::CUDAGuard g(logits.device());
  auto o32 = logits.options().dtype(torch::kFloat32);
  auto w = torch::empty({N, K}, o32);
  auto idx = torch::empty({N, K}, logits.options().dtype(torch::kInt32));
  auto counts = torch::zeros({E}, o32);
  auto psum = torch::zeros({E}, o32);
  if (N == 0) return {w, idx, counts, psum};
  auto st = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == torch::kBFloat16)
    router_fwd_kernel<__nv_bfloat16><<<warp_grid(N), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), N, E, K, norm, w.data_ptr<float>(),
        idx.data_ptr<int>(), counts.data_ptr<float>(), psum.data_ptr<float>(), error_flag_ptr());
  else
    router_fwd_kernel<float><<<warp_grid(N), 256, 0, st>>>(
        logits.data_ptr<float>(), N, E, K, norm, w.data_ptr<float>(), idx.data_ptr<int>(),
        counts.data_ptr<float>(), psum.data_ptr<float>(), error_flag_ptr());
  NQ_CHECK_CUDA(cudaGetLastError());
  return {w, idx, counts, psum};
}

torch::Tensor router_bwd(torch::Tensor logits, torch::Tensor w, torch::Tensor idx, torch::Tensor dw,
                         torch::Tensor dpsum, bool norm) {
  const int N = logits.size(0), E = logits.size(1), K = idx.size(1);
  c10::cuda::CUDAGuard g(logits.device());
  auto dl = torch::empty_like(logits);
  if (N == 0) return dl;
  auto st = at::cuda::getCurrentCUDAStream();
  auto dwc = dw.to(torch::kFloat32).contiguous();
  auto dpc = dpsum.to(torch::kFloat32).contiguous();
  if (logits.scalar_type() == torch::kBFloat16)
    router_bwd_kernel<__nv_bfloat16><<<warp_grid(N), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), w.data_ptr<float>(), idx.data_ptr<int>(),
        dwc.data_ptr<float>(), dpc.data_ptr<float>(), N, E, K, norm,
        reinterpret_cast<__nv_bfloat16*>(dl.data_ptr()));
  else
    router_bwd_kernel<float><<<warp_grid(N), 256, 0, st>>>(
        logits.data_ptr<float>(), w.data_ptr<float>(), idx.data_ptr<int>(), dwc.data_ptr<float>(),
        dpc.data_ptr<float>(), N, E, K, norm, dl.data_ptr<float>());
  NQ_CHECK_CUDA(cudaGetLastError());
  return dl;
}

// -------------------------------------------------------------- plan (sort)
constexpr int kChunk = 1024;

__global__ void plan_count_kernel(const int* __restrict__ idx, int64_t n, int E, int* __restrict__ chunk_cnt) {
  __shared__ int h[kMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kChunk;
  for (int i = threadIdx.x; i < kChunk; i += blockDim.x) {
    const int64_t j = base + i;
    if (j < n) atomicAdd(&h[idx[j]], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_cnt[static_cast<int64_t>(blockIdx.x) * E + e] = h[e];
}

// chunk_cnt [C, E] -> exclusive per-expert prefix over chunks (in place), offsets [E+1]
__global__ void plan_scan_kernel(int* __restrict__ chunk_cnt, int C, int E, int cap, int pad,
                                 int* __restrict__ offsets) {
  __shared__ int tot[kMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int c = 0; c < C; ++c) {
      const int v = chunk_cnt[static_cast<int64_t>(c) * E + e];
      chunk_cnt[static_cast<int64_t>(c) * E + e] = run;
      run += v;
    }
    tot[e] = (cap >= 0) ? min(run, cap) : run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = off;
      off += (tot[e] + pad - 1) / pad * pad;
    }
    offsets[E] = off;
  }
}

// Stable ranks inside each chunk (one warp walks its chunk in order).
__global__ void plan_assign_kernel(const int* __restrict__ idx, int64_t n, int E, int K, int cap,
                                   const int* __restrict__ chunk_base, const int* __restrict__ offsets,
                                   int* __restrict__ slot_of, int* __restrict__ src_of) {
  __shared__ int run[kMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) run[e] = 0;
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kChunk;
  for (int i0 = 0; i0 < kChunk; i0 += 32) {
    const int64_t j = base + i0 + lane;
    const bool valid = j < n;
    const int e = valid ? idx[j] : -1 - lane;  // unique dummy keys for invalid lanes
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int before = __popc(same & ((1u << lane) - 1u));
    int r = 0;
    if (valid) r = chunk_base[static_cast<int64_t>(blockIdx.x) * E + e] + run[e] + before;
    __syncwarp();
    if (valid && (same >> lane) == 1u) run[e] += __popc(same);  // highest lane of the group
    __syncwarp();
    if (valid) {
      if (cap < 0 || r < cap) {
        const int slot = offsets[e] + r;
        slot_of[j] = slot;
        src_of[slot] = static_cast<int>(j / K);
      } else {
        slot_of[j] = -1;
      }
    }
  }
}

std::vector<torch::Tensor> moe_plan(torch::Tensor idx, int64_t E, int64_t cap, int64_t pad) {
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && idx.is_contiguous() && E <= kMaxE, "moe_plan: idx int32");
  TORCH_CHECK(pad >= 1, "moe_plan: pad (segment alignment) must be >= 1");
  const int N = idx.size(0), K = idx.size(1);
  const int64_t n = static_cast<int64_t>(N) * K;
  const int64_t rows_cap = n + E * pad;
  c10::cuda::CUDAGuard g(idx.device());
  auto oi = idx.options();
  auto slot_of = torch::empty({N, K}, oi);
  auto offsets = torch::empty({E + 1}, oi);
  auto src_of = torch::full({rows_cap}, -1, oi);
  if (n == 0) { offsets.zero_(); return {slot_of, offsets, src_of}; }
  const int C = static_cast<int>((n + kChunk - 1) / kChunk);
  auto chunk = torch::empty({C, E}, oi);
  auto st = at::cuda::getCurrentCUDAStream();
  plan_count_kernel<<<C, 256, 0, st>>>(idx.data_ptr<int>(), n, E, chunk.data_ptr<int>());
  plan_scan_kernel<<<1, 256, 0, st>>>(chunk.data_ptr<int>(), C, E, static_cast<int>(cap), static_cast<int>(pad), offsets.data_ptr<int>());
  plan_assign_kernel<<<C, 64, 0, st>>>(idx.data_ptr<int>(), n, E, K, static_cast<int>(cap), chunk.data_ptr<int>(),
                                       offsets.data_ptr<int>(), slot_of.data_ptr<int>(), src_of.data_ptr<int>());
  NQ_CHECK_CUDA(cudaGetLastError());
  return {slot_of, offsets, src_of};
}

// ------------------------------------------------------- gather / combine
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ src,
                                   __nv_bfloat16* __restrict__ out, int64_t R, int H) {
  const int H8 = H / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < R * H8; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / H8;
    const int c = static_cast<int>(v - r * H8);
    const int s = src[r];
    uint4 val = make_uint4(0, 0, 0, 0);
    if (s >= 0) val = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(s) * H)[c];
    reinterpret_cast<uint4*>(out + r * H)[c] = val;
  }
}

// out[t] = sum_j w[t,j] * y[slot[t,j]]
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ slot,
                               const float* __restrict__ w, __nv_bfloat16* __restrict__ out, int N,
                               int K, int H) {
  const int H8 = H / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < (int64_t)N * H8; v += (int64_t)gridDim.x * blockDim.x) {
    const int t = static_cast<int>(v / H8);
    const int c = static_cast<int>(v - static_cast<int64_t>(t) * H8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < K; ++j) {
      const int s = slot[static_cast<int64_t>(t) * K + j];
      if (s < 0) continue;
      const float wj = w[static_cast<int64_t>(t) * K + j];
      float f[8];
      load8(y + static_cast<int64_t>(s) * H + c, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += wj * f[i];
    }
    store8(out + static_cast<int64_t>(t) * H + c, acc);
  }
}

// dy[slot[t,j]] = w[t,j] * dout[t];  dw[t,j] = <dout[t], y[slot[t,j]]>   (warp per (t, j))
__global__ void combine_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ y,
                                   const int* __restrict__ slot, const float* __restrict__ w,
                                   __nv_bfloat16* __restrict__ dy, float* __restrict__ dw, int N, int K, int H) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int64_t it = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; it < (int64_t)N * K; it += warps) {
    const int64_t t = it / K;
    const int s = slot[it];
    if (s < 0) { if (lane == 0) dw[it] = 0.f; continue; }
    const float wj = w[it];
    float dot = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      float d[8], yy[8], o[8];
      load8(dout + t * H + c, d);
      load8(y + static_cast<int64_t>(s) * H + c, yy);
#pragma unroll
      for (int i = 0; i < 8; ++i) { dot += d[i] * yy[i]; o[i] = wj * d[i]; }
      store8(dy + static_cast<int64_t>(s) * H + c, o);
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[it] = dot;
  }
}

// dx[t] = sum_j dxp[slot[t,j]]
__global__ void scatter_add_kernel(const __nv_bfloat16* __restrict__ dxp, const int* __restrict__ slot,
                                   __nv_bfloat16* __restrict__ dx, int N, int K, int H) {
  const int H8 = H / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < (int64_t)N * H8; v += (int64_t)gridDim.x * blockDim.x) {
    const int t = static_cast<int>(v / H8);
    const int c = static_cast<int>(v - static_cast<int64_t>(t) * H8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < K; ++j) {
      const int s = slot[static_cast<int64_t>(t) * K + j];
      if (s < 0) continue;
      float f[8];
      load8(dxp + static_cast<int64_t>(s) * H + c, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += f[i];
    }
    store8(dx + static_cast<int64_t>(t) * H + c, acc);
  }
}

static int rows_grid(int64_t n) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, num_sms() * 16)));
}

torch::Tensor moe_gather(torch::Tensor x, torch::Tensor src_of) {
  check_bf16(x, "x");
  TORCH_CHECK(x.is_contiguous() && x.size(1) % 8 == 0, "moe_gather: x [N,H], H % 8");
  const int64_t R = src_of.numel();
  const int H = x.size(1);
  c10::cuda::CUDAGuard g(x.device());
  auto out = torch::empty({R, H}, x.options());
  if (R == 0) return out;
  gather_rows_kernel<<<rows_grid(R * H / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), src_of.data_ptr<int>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), R, H);
  NQ_CHECK_CUDA(cudaGetLastError());
  return out;
}

torch::Tensor moe_combine(torch::Tensor y, torch::Tensor slot, torch::Tensor w) {
  check_bf16(y, "y");
  const int N = slot.size(0), K = slot.size(1), H = y.size(1);
  c10::cuda::CUDAGuard g(y.device());
  auto out = torch::empty({N, H}, y.options());
  if (N == 0) return out;
  auto wc = w.to(torch::kFloat32).contiguous();
  combine_kernel<<<rows_grid((int64_t)N * H / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), slot.data_ptr<int>(), wc.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), N, K, H);
  NQ_CHECK_CUDA(cudaGetLastError());
  return out;
}

std::vector<torch::Tensor> moe_combine_bwd(torch::Tensor dout, torch::Tensor y, torch::Tensor slot, torch::Tensor w) {
  check_bf16(dout, "dout"); check_bf16(y, "y");
  const int N = slot.size(0), K = slot.size(1), H = y.size(1);
  c10::cuda::CUDAGuard g(y.device());
  auto dy = torch::zeros_like(y);
  auto dw = torch::empty({N, K}, y.options().dtype(torch::kFloat32));
  if (N == 0) return {dy, dw};
  auto wc = w.to(torch::kFloat32).contiguous();
  combine_bwd_kernel<<<warp_grid((int64_t)N * K), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.contiguous().data_ptr()), reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()),
      slot.data_ptr<int>(), wc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dy.data_ptr()),
      dw.data_ptr<float>(), N, K, H);
  NQ_CHECK_CUDA(cudaGetLastError());
  return {dy, dw};
}

torch::Tensor moe_scatter_add(torch::Tensor dxp, torch::Tensor slot, int64_t N) {
  check_bf16(dxp, "dxp");
  const int K = slot.size(1), H = dxp.size(1);
  c10::cuda::CUDAGuard g(dxp.device());
  auto dx = torch::empty({N, H}, dxp.options());
  if (N == 0) return dx;
  scatter_add_kernel<<<rows_grid(N * H / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dxp.data_ptr()), slot.data_ptr<int>(),
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), N, K, H);
  NQ_CHECK_CUDA(cudaGetLastError());
  return dx;
}

}  // namespace nq
