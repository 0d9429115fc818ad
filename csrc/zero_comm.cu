// Data-parallel optimizer step over NVLink peer memory (ZeRO-2 without NCCL
// for the bulk traffic).
//
// Every rank's flat fp32 gradient buffer, bf16 compute copy and a small flag
// block live in symmetric memory (mapped into every peer's address space).
// Rank r owns the shard [b_r, e_r) of the flat buffers.  One optimizer step is
// three kernels on the compute stream plus one scalar all-reduce:
//
//  1. zero_rs_kernel: signals "gradients final" to every peer, waits (bounded)
//     until every peer has signalled, then reads its shard of every peer's
//     gradient buffer with 16-byte P2P loads, writes the mean into its own
//     buffer and accumulates the squared norm of the mean (for clipping).
//     This is the reduce-scatter, fused with the 1/world scale and the norm.
//  2. (host) all-reduce of the 4-byte squared norm, clip factor on the device.
//  3. zero_adamw_ag_kernel: AdamW on the shard, then the rounded bf16 values
//     are stored straight into every peer's compute copy (P2P stores): the
//     all-gather is fused into the optimizer.
//  4. zero_publish_kernel: signals "parameters published" and waits (bounded)
//     for every peer's signal, so the next forward reads complete weights.
//
// Flags follow the protocol of peer.cuh (release/acquire at system scope,
// bounded waits that record kErrTimeoutPeer and return).  No TMA or multicast
// is involved.
#include "common.cuh"
#include "peer.cuh"
#include "tmap.h"

namespace nq {

constexpr int kZeroMaxPeers = 8;

struct ZeroPeers {
  float* grad[kZeroMaxPeers];
  __nv_bfloat16* comp[kZeroMaxPeers];
  unsigned* flags[kZeroMaxPeers];  // [2 slots][kZeroMaxPeers sources] per rank
  int world;
  int rank;
};

// Thread t < world writes `epoch` into slot `slot`, source `rank`, of rank t's flags.
__device__ __forceinline__ void signal_peers(const ZeroPeers& P, int slot, unsigned epoch) {
  const int t = threadIdx.x;
  if (t < P.world) {
    __threadfence_system();
    st_release_sys(P.flags[t] + slot * kZeroMaxPeers + P.rank, epoch);
  }
}

// Whole block: wait until every source has reached `epoch` in our own slot.
__device__ __forceinline__ bool wait_peers(const ZeroPeers& P, int slot, unsigned epoch, int* err) {
  return block_wait_flags(P.flags[P.rank] + slot * kZeroMaxPeers, P.world, epoch, err);
}

__device__ __forceinline__ float4 ldcg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

template <int W>
__global__ void __launch_bounds__(256) zero_rs_kernel(ZeroPeers P, int64_t b, int64_t e, float inv,
                                                      float* __restrict__ sq_out, unsigned epoch,
                                                      int* err) {
  // Every block signals (idempotent), so whichever blocks are resident first
  // can never wait on a signal that only a not-yet-scheduled block would send.
  signal_peers(P, 0, epoch);
  if (!wait_peers(P, 0, epoch, err)) return;
  const float* src[W];
#pragma unroll
  for (int r = 0; r < W; ++r) src[r] = P.grad[r];
  float* dst = P.grad[P.rank];
  float sq = 0.f;
  const int64_t n4 = (e - b) / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // two 16-byte vectors per thread and iteration: 2*W independent loads in flight
  for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < n4; q += 2 * stride) {
    const int64_t i0 = b + q * 4;
    const bool two = q + stride < n4;
    const int64_t i1 = b + (q + stride) * 4;
    float4 a[W], c[W];
#pragma unroll
    for (int r = 0; r < W; ++r) {
      a[r] = ldcg4(src[r] + i0);
      if (two) c[r] = ldcg4(src[r] + i1);
    }
    float4 s0 = a[0], s1 = c[0];
#pragma unroll
    for (int r = 1; r < W; ++r) {
      s0.x += a[r].x; s0.y += a[r].y; s0.z += a[r].z; s0.w += a[r].w;
      if (two) { s1.x += c[r].x; s1.y += c[r].y; s1.z += c[r].z; s1.w += c[r].w; }
    }
    s0.x *= inv; s0.y *= inv; s0.z *= inv; s0.w *= inv;
    *reinterpret_cast<float4*>(dst + i0) = s0;
    sq += s0.x * s0.x + s0.y * s0.y + s0.z * s0.z + s0.w * s0.w;
    if (two) {
      s1.x *= inv; s1.y *= inv; s1.z *= inv; s1.w *= inv;
      *reinterpret_cast<float4*>(dst + i1) = s1;
      sq += s1.x * s1.x + s1.y * s1.y + s1.z * s1.z + s1.w * s1.w;
    }
  }
  __shared__ float red[32];
  sq = block_sum(sq, red);
  if (threadIdx.x == 0) atomicAdd(sq_out, sq);
}

// clip = min(1, max_norm / (sqrt(sq) + 1e-6)); norm = sqrt(sq)
__global__ void zero_clip_kernel(const float* __restrict__ sq, float max_norm, float* __restrict__ clip,
                                 float* __restrict__ norm) {
  const float n = sqrtf(*sq);
  *norm = n;
  *clip = max_norm > 0.f ? fminf(1.f, max_norm / (n + 1e-6f)) : 1.f;
}

template <int W>
__global__ void __launch_bounds__(256) zero_adamw_ag_kernel(
    ZeroPeers P, float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
    const float* __restrict__ clip, int64_t begin, int64_t end, int64_t sbase, int64_t decay_end,
    float lr_d, float lr_n, float b1, float b2, float eps, float wd, float bc1, float bc2) {
  // m / v cover flat elements [sbase, ...): the shard (sbase = begin) or all
  m -= sbase;
  v -= sbase;
  const float* g = P.grad[P.rank];
  const float cs = *clip;
  const float rbc1 = 1.f / bc1, rbc2 = 1.f / bc2;
  __nv_bfloat16* dst[W];
#pragma unroll
  for (int r = 0; r < W; ++r) dst[r] = P.comp[r];
  const int64_t n4 = (end - begin) / 4;
  for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < n4;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = begin + q * 4;
    const bool decay = i < decay_end;
    const float lr = decay ? lr_d : lr_n;
    const float w = decay ? wd : 0.f;
    float4 pv = *reinterpret_cast<float4*>(p + i);
    const float4 gv = *reinterpret_cast<const float4*>(g + i);
    float4 mv = *reinterpret_cast<float4*>(m + i);
    float4 vv = *reinterpret_cast<float4*>(v + i);
    float* pp = &pv.x;
    const float* gg = &gv.x;
    float* mm = &mv.x;
    float* vq = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gr = gg[k] * cs;
      const float x = pp[k] * (1.f - lr * w);
      mm[k] = b1 * mm[k] + (1.f - b1) * gr;
      vq[k] = b2 * vq[k] + (1.f - b2) * gr * gr;
      const float denom = sqrtf(vq[k] * rbc2) + eps;
      pp[k] = x - lr * (mm[k] * rbc1) / denom;
    }
    *reinterpret_cast<float4*>(p + i) = pv;
    *reinterpret_cast<float4*>(m + i) = mv;
    *reinterpret_cast<float4*>(v + i) = vv;
    __nv_bfloat162 lo = __floats2bfloat162_rn(pv.x, pv.y), hi = __floats2bfloat162_rn(pv.z, pv.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
#pragma unroll
    for (int r = 0; r < W; ++r) *reinterpret_cast<uint2*>(dst[r] + i) = u;
  }
  __threadfence_system();
}

__global__ void zero_publish_kernel(ZeroPeers P, unsigned epoch, int* err) {
  signal_peers(P, 1, epoch);
  wait_peers(P, 1, epoch, err);
}

// --------------------------------------------------------------------- host
static ZeroPeers make_peers(const std::vector<int64_t>& grad, const std::vector<int64_t>& comp,
                            const std::vector<int64_t>& flags, int64_t rank) {
  const int world = static_cast<int>(grad.size());
  TORCH_CHECK(world >= 1 && world <= kZeroMaxPeers, "zero_comm: 1..8 ranks");
  TORCH_CHECK(comp.size() == grad.size() && flags.size() == grad.size(), "zero_comm: pointer lists");
  TORCH_CHECK(rank >= 0 && rank < world, "zero_comm: rank");
  ZeroPeers P{};
  for (int r = 0; r < world; ++r) {
    P.grad[r] = reinterpret_cast<float*>(grad[r]);
    P.comp[r] = reinterpret_cast<__nv_bfloat16*>(comp[r]);
    P.flags[r] = reinterpret_cast<unsigned*>(flags[r]);
    TORCH_CHECK(grad[r] % 16 == 0 && comp[r] % 8 == 0 && flags[r] % 4 == 0, "zero_comm: alignment");
  }
  P.world = world;
  P.rank = static_cast<int>(rank);
  return P;
}

#define NQ_W_DISPATCH(W, ...)                                      \
  switch (W) {                                                     \
    case 1: { constexpr int WW = 1; __VA_ARGS__; break; }          \
    case 2: { constexpr int WW = 2; __VA_ARGS__; break; }          \
    case 4: { constexpr int WW = 4; __VA_ARGS__; break; }          \
    case 8: { constexpr int WW = 8; __VA_ARGS__; break; }          \
    default: TORCH_CHECK(false, "zero_comm: world size must be 1, 2, 4 or 8"); \
  }

// Reduce-scatter of the mean gradient into this rank's shard, fused with the
// squared-norm partial (added into sq_out).  grid_ctas = 0 picks 3 per SM.
// scale multiplies the mean (expert spans: the sum over the ranks holding the
// same experts divided by the whole data-parallel world).
void zero_rs(std::vector<int64_t> grad, std::vector<int64_t> comp, std::vector<int64_t> flags,
             int64_t rank, int64_t begin, int64_t end, torch::Tensor sq_out, int64_t epoch,
             int64_t grid_ctas, double scale) {
  auto P = make_peers(grad, comp, flags, rank);
  TORCH_CHECK(begin % 4 == 0 && end % 4 == 0 && end >= begin, "zero_rs: 4-aligned shard");
  TORCH_CHECK(sq_out.scalar_type() == torch::kFloat32 && sq_out.is_cuda(), "zero_rs: sq_out fp32");
  auto st = at::cuda::getCurrentCUDAStream();
  const int grid = grid_ctas > 0 ? static_cast<int>(grid_ctas) : 3 * num_sms();
  NQ_W_DISPATCH(P.world, zero_rs_kernel<WW><<<grid, 256, 0, st>>>(
      P, begin, end, static_cast<float>(scale) / P.world, sq_out.data_ptr<float>(), static_cast<unsigned>(epoch),
      error_flag_ptr()));
  NQ_CHECK_CUDA(cudaGetLastError());
}

void zero_clip(torch::Tensor sq, double max_norm, torch::Tensor clip, torch::Tensor norm) {
  auto st = at::cuda::getCurrentCUDAStream();
  zero_clip_kernel<<<1, 1, 0, st>>>(sq.data_ptr<float>(), static_cast<float>(max_norm),
                                     clip.data_ptr<float>(), norm.data_ptr<float>());
  NQ_CHECK_CUDA(cudaGetLastError());
}

void zero_adamw_ag(std::vector<int64_t> grad, std::vector<int64_t> comp, std::vector<int64_t> flags,
                   int64_t rank, torch::Tensor master, torch::Tensor m, torch::Tensor v,
                   torch::Tensor clip, int64_t begin, int64_t end, int64_t sbase, int64_t decay_end,
                   double lr_d, double lr_n, double b1, double b2, double eps, double wd, double bc1,
                   double bc2) {
  auto P = make_peers(grad, comp, flags, rank);
  TORCH_CHECK(begin % 4 == 0 && end % 4 == 0 && end >= begin && sbase % 4 == 0, "zero_adamw_ag: 4-aligned shard");
  TORCH_CHECK(sbase <= begin && end - sbase <= m.numel() && m.numel() == v.numel(),
              "zero_adamw_ag: optimizer state does not cover the shard");
  auto st = at::cuda::getCurrentCUDAStream();
  const int64_t n4 = (end - begin) / 4;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n4 + 255) / 256, num_sms() * 8)));
  NQ_W_DISPATCH(P.world, zero_adamw_ag_kernel<WW><<<grid, 256, 0, st>>>(
      P, master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), clip.data_ptr<float>(),
      begin, end, sbase, decay_end, (float)lr_d, (float)lr_n, (float)b1, (float)b2, (float)eps, (float)wd,
      (float)bc1, (float)bc2));
  NQ_CHECK_CUDA(cudaGetLastError());
}

void zero_publish(std::vector<int64_t> grad, std::vector<int64_t> comp, std::vector<int64_t> flags,
                  int64_t rank, int64_t epoch) {
  auto P = make_peers(grad, comp, flags, rank);
  auto st = at::cuda::getCurrentCUDAStream();
  zero_publish_kernel<<<1, 32, 0, st>>>(P, static_cast<unsigned>(epoch), error_flag_ptr());
  NQ_CHECK_CUDA(cudaGetLastError());
}

}  // namespace nq
