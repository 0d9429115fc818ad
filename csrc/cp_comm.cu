// Context-parallel K/V exchange over NVLink peer memory.
//
// Forward: cp_kv_scatter_kernel stores each local token's rotated k row and its
// v row into every rank's gathered key/value buffer at the token's global
// position (P2P stores: the all-gather and the zigzag-to-natural reordering in
// one pass) and the last block publishes a flag; the attention forward kernel
// (attn_fwd_cp with flags) waits for the owner's flag before its TMA loads a
// key block, so keys from early ranks are consumed while later ones land.
// Backward: every rank's attention backward writes its partial dk|dv for all
// gathered keys into its own buffer and publishes a flag; cp_dkv_gather_kernel
// waits for every rank and sums, for each local token, the partials of the
// token's position from every rank (P2P loads: the reduce-scatter).
// Flags follow peer.cuh.  Flag block per rank: [2 channels][8 sources]:
// 0 = keys/values published, 1 = dk/dv partials published.
#include "common.cuh"
#include "peer.cuh"
#include "tmap.h"

namespace nq {

constexpr int kCPMax = 8;

struct CPPeers {
  void* buf[kCPMax];        // per rank: gathered kv (bf16) or dkv partials (fp32)
  unsigned* flags[kCPMax];
  int world, rank;
};

static CPPeers make_cp(const std::vector<int64_t>& buf, const std::vector<int64_t>& flags, int64_t rank) {
  CPPeers P{};
  P.world = static_cast<int>(flags.size());
  TORCH_CHECK(P.world >= 1 && P.world <= kCPMax && buf.size() == flags.size(), "cp: 1..8 ranks");
  P.rank = static_cast<int>(rank);
  for (int r = 0; r < P.world; ++r) {
    P.buf[r] = reinterpret_cast<void*>(buf[r]);
    P.flags[r] = reinterpret_cast<unsigned*>(flags[r]);
  }
  return P;
}

// One warp per local token: kv row = [k (Hk*D) | v (Hk*D)] -> every rank's
// buffer at row b*Sk + pos[t].
__global__ void cp_kv_scatter_kernel(CPPeers P, const __nv_bfloat16* __restrict__ qk,
                                     const __nv_bfloat16* __restrict__ qkv, const int64_t* __restrict__ pos,
                                     int T, int S, int Sk, int Hq, int Hk, int D, unsigned seq,
                                     unsigned* counter, unsigned target) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int KD8 = Hk * D / 8;
  for (int t = gw; t < T; t += warps) {
    const int b = t / S;
    const int64_t row = static_cast<int64_t>(b) * Sk + pos[t];
    const uint4* ks = reinterpret_cast<const uint4*>(qk + (static_cast<int64_t>(t) * (Hq + Hk) + Hq) * D);
    const uint4* vs = reinterpret_cast<const uint4*>(qkv + (static_cast<int64_t>(t) * (Hq + 2 * Hk) + Hq + Hk) * D);
    for (int c = lane; c < KD8; c += 32) {
      const uint4 kv = ks[c], vv = vs[c];
#pragma unroll
      for (int r = 0; r < kCPMax; ++r) {
        if (r >= P.world) break;
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(P.buf[r]) + row * 2 * Hk * D);
        dst[c] = kv;
        dst[KD8 + c] = vv;
      }
    }
  }
  grid_done_signal(counter, target, P.flags, 0 * kCPMax + P.rank, P.world, seq);
}

// One warp per local token: out[t] = sum_r dkv_r[b*Sk + pos[t]] (fp32 rows of
// 2*Hk*D), after every rank published its partials (channel 1).
__global__ void cp_dkv_gather_kernel(CPPeers P, const int64_t* __restrict__ pos, float* __restrict__ out, int T,
                                     int S, int Sk, int W2, unsigned seq, int* err) {
  if (!block_wait_flags(P.flags[P.rank] + 1 * kCPMax, P.world, seq, err)) return;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int n4 = W2 / 4;
  for (int t = gw; t < T; t += warps) {
    const int b = t / S;
    const int64_t row = static_cast<int64_t>(b) * Sk + pos[t];
    for (int c = lane; c < n4; c += 32) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < P.world; ++r) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(P.buf[r]) + row * W2) + c);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      reinterpret_cast<float4*>(out + static_cast<int64_t>(t) * W2)[c] = acc;
    }
  }
}

// Publish channel `ch` to every rank (stream order makes the previous
// kernels' stores complete).
__global__ void cp_signal_kernel(CPPeers P, int ch, unsigned seq) {
  if (threadIdx.x < P.world) {
    __threadfence_system();
    st_release_sys(P.flags[threadIdx.x] + ch * kCPMax + P.rank, seq);
  }
}

// ---------------------------------------------------------------------- host
int64_t cp_kv_scatter(std::vector<int64_t> kv_bufs, std::vector<int64_t> flags, int64_t rank, torch::Tensor qk,
                      torch::Tensor qkv, torch::Tensor pos, int64_t B, int64_t S, int64_t Sk, int64_t Hq, int64_t Hk,
                      int64_t D, int64_t seq, torch::Tensor counter, int64_t counter_before) {
  auto P = make_cp(kv_bufs, flags, rank);
  TORCH_CHECK(pos.scalar_type() == torch::kInt64 && pos.numel() == B * S, "cp_kv_scatter: pos int64 [B*S]");
  TORCH_CHECK((Hk * D) % 8 == 0, "cp_kv_scatter: Hk*D % 8");
  const int T = static_cast<int>(B * S);
  const int grid = std::max(1, std::min((T + 7) / 8, num_sms() * 8));
  cp_kv_scatter_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      P, reinterpret_cast<const __nv_bfloat16*>(qk.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
      pos.data_ptr<int64_t>(), T, static_cast<int>(S), static_cast<int>(Sk), static_cast<int>(Hq),
      static_cast<int>(Hk), static_cast<int>(D), static_cast<unsigned>(seq),
      reinterpret_cast<unsigned*>(counter.data_ptr()), static_cast<unsigned>(counter_before + grid));
  NQ_CHECK_CUDA(cudaGetLastError());
  return grid;
}

void cp_signal(std::vector<int64_t> bufs, std::vector<int64_t> flags, int64_t rank, int64_t ch, int64_t seq) {
  auto P = make_cp(bufs, flags, rank);
  cp_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(P, static_cast<int>(ch), static_cast<unsigned>(seq));
  NQ_CHECK_CUDA(cudaGetLastError());
}

torch::Tensor cp_dkv_gather(std::vector<int64_t> dkv_bufs, std::vector<int64_t> flags, int64_t rank, torch::Tensor pos,
                            int64_t B, int64_t S, int64_t Sk, int64_t W2, int64_t seq) {
  auto P = make_cp(dkv_bufs, flags, rank);
  TORCH_CHECK(W2 % 4 == 0, "cp_dkv_gather: width % 4");
  const int T = static_cast<int>(B * S);
  auto out = torch::empty({T, W2}, pos.options().dtype(torch::kFloat32));
  const int grid = std::max(1, std::min((T + 7) / 8, num_sms() * 8));
  cp_dkv_gather_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      P, pos.data_ptr<int64_t>(), out.data_ptr<float>(), T, static_cast<int>(S), static_cast<int>(Sk),
      static_cast<int>(W2), static_cast<unsigned>(seq), error_flag_ptr());
  NQ_CHECK_CUDA(cudaGetLastError());
  return out;
}

}  // namespace nq
