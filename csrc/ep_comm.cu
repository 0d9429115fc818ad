// Expert-parallel dispatch and combine over NVLink peer memory.
//
// Each rank routes its N tokens to E experts (top-k); rank d owns experts
// [d*El, (d+1)*El).  Every rank has, in symmetric memory, a receive buffer laid
// out exactly as its grouped expert GEMMs want it: one 128-row-aligned segment
// per local expert, and inside a segment the rows of source rank 0, then rank
// 1, ... in each source's token order.  Because every rank learns every
// rank's per-expert counts (ep_layout_kernel), each source computes the exact
// destination row of each (token, slot) pair and stores the token's row there
// itself (ep_dispatch_kernel: the all-to-all is a scatter of P2P stores fused
// with the permutation).  After the experts ran, each source pulls its pairs'
// output rows back with P2P loads and forms the weighted top-k sum
// (ep_combine_kernel).  The backward mirrors both: the weighted output
// gradient is pushed into the experts' gradient buffer, and the input gradient
// is pulled and summed over the k slots.
//
// No host synchronisation: counts, layout and segment offsets stay on the
// device; the receive capacity is a fixed bound and an overflowing pair is
// dropped with an error code rather than written out of bounds.  Flags follow
// peer.cuh (monotonic sequence numbers, bounded waits).  Flag block per rank:
// [8 channels][8 sources]; channels: 0 counts, 1 dispatch, 2 expert outputs,
// 3 output gradients, 4 input gradients.
#include "common.cuh"
#include "peer.cuh"
#include "tmap.h"

namespace nq {

constexpr int kEPMax = 8;
constexpr int kEPMaxE = 256;

struct EPPeers {
  unsigned* flags[kEPMax];
  int* counts[kEPMax];          // [W][E] per rank: counts[src][e] of tokens src routes to e
  __nv_bfloat16* buf[kEPMax];   // the exchanged row buffer of each rank (role set per launch)
  int world, rank;
};

static EPPeers make_ep(const std::vector<int64_t>& flags, const std::vector<int64_t>& counts,
                       const std::vector<int64_t>& buf, int64_t rank) {
  EPPeers P{};
  P.world = static_cast<int>(flags.size());
  TORCH_CHECK(P.world >= 1 && P.world <= kEPMax, "ep: 1..8 ranks");
  TORCH_CHECK(counts.size() == flags.size() && (buf.empty() || buf.size() == flags.size()), "ep: pointer lists");
  P.rank = static_cast<int>(rank);
  for (int r = 0; r < P.world; ++r) {
    P.flags[r] = reinterpret_cast<unsigned*>(flags[r]);
    P.counts[r] = reinterpret_cast<int*>(counts[r]);
    P.buf[r] = buf.empty() ? nullptr : reinterpret_cast<__nv_bfloat16*>(buf[r]);
  }
  return P;
}

// One CTA.  Publishes this rank's per-expert counts to every rank, waits for
// everyone's, then computes
//   dest_base[e]  : first row of this rank's pairs for expert e in the owner's buffer
//   seg_off[j]    : start of local expert j's segment (j <= El), 128-aligned
//   seg_used[j]   : rows of local expert j actually filled
__global__ void ep_layout_kernel(EPPeers P, const float* __restrict__ counts_local, int E, int El,
                                 unsigned seq, int* __restrict__ dest_base, int* __restrict__ seg_off,
                                 int* __restrict__ seg_used, int cap, int* err) {
  __shared__ int s_tot[kEPMaxE];
  __shared__ int s_seg[kEPMaxE + 1];
  const int W = P.world;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int c = static_cast<int>(counts_local[e] + 0.5f);
    for (int r = 0; r < W; ++r) P.counts[r][P.rank * E + e] = c;
  }
  __syncthreads();
  if (threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(P.flags[threadIdx.x] + 0 * kEPMax + P.rank, seq);
  }
  if (!block_wait_flags(P.flags[P.rank] + 0 * kEPMax, W, seq, err)) return;
  const int* all = P.counts[P.rank];  // [W][E], local copy of everyone's counts
  // total rows per global expert
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t = 0;
    for (int s = 0; s < W; ++s) t += all[s * E + e];
    s_tot[e] = t;
  }
  __syncthreads();
  // segment starts of every owner's experts (each owner's layout starts at 0)
  if (threadIdx.x < W) {
    const int d = threadIdx.x;
    int off = 0;
    for (int j = 0; j < El; ++j) {
      s_seg[d * El + j] = off;
      off += (s_tot[d * El + j] + 127) / 128 * 128;
    }
    if (d == P.rank) s_seg[E] = off;  // end of this rank's used region
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int pre = 0;
    for (int s = 0; s < P.rank; ++s) pre += all[s * E + e];
    dest_base[e] = s_seg[e] + pre;
  }
  for (int j = threadIdx.x; j <= El; j += blockDim.x) {
    const int v = (j < El) ? s_seg[P.rank * El + j] : s_seg[E];
    seg_off[j] = min(v, cap);
    if (j < El) seg_used[j] = s_tot[P.rank * El + j];
  }
  if (threadIdx.x == 0 && s_seg[E] > cap) atomicCAS(err, 0, kErrBadArg);
}

// One warp per (token, slot) pair: the token's row goes to its expert owner's
// buffer at dest_base[e] + (index of the pair among this rank's pairs for e).
// Also zeroes the padding rows of this rank's own buffer, and records each
// pair's destination row for the combine.
__global__ void ep_dispatch_kernel(EPPeers P, const __nv_bfloat16* __restrict__ x, const int* __restrict__ idx,
                                   const int* __restrict__ slot_of, const int* __restrict__ loc_off,
                                   const int* __restrict__ dest_base, const int* __restrict__ seg_off,
                                   const int* __restrict__ seg_used, int* __restrict__ dest_row, int N, int K,
                                   int H, int El, int cap, unsigned seq, unsigned* counter, unsigned target,
                                   int* err) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int H8 = H / 8;
  const int64_t pairs = static_cast<int64_t>(N) * K;
  for (int64_t p = gw; p < pairs; p += warps) {
    const int t = static_cast<int>(p / K);
    const int e = idx[p];
    const int d = e / El;
    const int row = dest_base[e] + (slot_of[p] - loc_off[e]);
    if (row < 0 || row >= cap) {
      if (lane == 0) { atomicCAS(err, 0, kErrBadArg); dest_row[p] = -1; }
      continue;
    }
    if (lane == 0) dest_row[p] = row;
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * H);
    uint4* dst = reinterpret_cast<uint4*>(P.buf[d] + static_cast<int64_t>(row) * H);
    for (int c = lane; c < H8; c += 32) dst[c] = src[c];
  }
  // padding rows of this rank's own segments
  uint4* own = reinterpret_cast<uint4*>(P.buf[P.rank]);
  for (int j = 0; j < El; ++j) {
    const int64_t lo = seg_off[j] + seg_used[j], hi = seg_off[j + 1];
    for (int64_t v = (lo * H8) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < hi * H8;
         v += (int64_t)gridDim.x * blockDim.x)
      own[v] = make_uint4(0, 0, 0, 0);
  }
  grid_done_signal(counter, target, P.flags, 1 * kEPMax + P.rank, P.world, seq);
}

// Whole grid: wait until every rank has published `seq` on channel `ch` here.
__global__ void ep_wait_kernel(EPPeers P, int ch, unsigned seq, int* err) {
  block_wait_flags(P.flags[P.rank] + ch * kEPMax, P.world, seq, err);
}

// Publish `seq` on channel `ch` of every rank (after this rank's previous
// kernels, which stream order has completed).
__global__ void ep_signal_kernel(EPPeers P, int ch, unsigned seq) {
  if (threadIdx.x < P.world) {
    __threadfence_system();
    st_release_sys(P.flags[threadIdx.x] + ch * kEPMax + P.rank, seq);
  }
}

// out[t] = sum_s w[t,s] * y_owner[dest_row[t,s]]; the pulled rows are kept in
// y_pulled[t*K+s] for the backward (weights' gradient).  Waits for channel 2.
__global__ void ep_combine_kernel(EPPeers P, const int* __restrict__ idx, const int* __restrict__ dest_row,
                                  const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                  __nv_bfloat16* __restrict__ y_pulled, int N, int K, int H, int El,
                                  unsigned seq, int* err) {
  if (!block_wait_flags(P.flags[P.rank] + 2 * kEPMax, P.world, seq, err)) return;
  const int H8 = H / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < static_cast<int64_t>(N) * H8;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int t = static_cast<int>(v / H8);
    const int c = static_cast<int>(v - static_cast<int64_t>(t) * H8);
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int s = 0; s < K; ++s) {
      const int64_t p = static_cast<int64_t>(t) * K + s;
      const int row = dest_row[p];
      uint4 u = make_uint4(0, 0, 0, 0);
      if (row >= 0) {
        const int d = idx[p] / El;
        u = __ldcg(reinterpret_cast<const uint4*>(P.buf[d] + static_cast<int64_t>(row) * H) + c);
      }
      reinterpret_cast<uint4*>(y_pulled + p * H)[c] = u;
      const float ws = w[p];
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(hv[i]);
        acc[2 * i] += ws * f.x;
        acc[2 * i + 1] += ws * f.y;
      }
    }
    store8(out + static_cast<int64_t>(t) * H + c * 8, acc);
  }
}

// Backward of the combine: pushes w[t,s] * dout[t] into the owner's gradient
// buffer at dest_row[t,s] and computes dw[t,s] = <dout[t], y_pulled[t,s]>.
// One warp per pair; publishes channel 3 when the grid is done.
__global__ void ep_combine_bwd_kernel(EPPeers P, const int* __restrict__ idx, const int* __restrict__ dest_row,
                                      const float* __restrict__ w, const __nv_bfloat16* __restrict__ dout,
                                      const __nv_bfloat16* __restrict__ y_pulled, float* __restrict__ dw, int N,
                                      int K, int H, int El, unsigned seq, unsigned* counter, unsigned target) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int H8 = H / 8;
  const int64_t pairs = static_cast<int64_t>(N) * K;
  for (int64_t p = gw; p < pairs; p += warps) {
    const int t = static_cast<int>(p / K);
    const int row = dest_row[p];
    const float ws = w[p];
    const int d = idx[p] / El;
    float dot = 0.f;
    for (int c = lane; c < H8; c += 32) {
      float g[8], y[8], o[8];
      load8(dout + static_cast<int64_t>(t) * H + c * 8, g);
      load8(y_pulled + p * H + c * 8, y);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dot += g[i] * y[i];
        o[i] = g[i] * ws;
      }
      if (row >= 0) store8(P.buf[d] + static_cast<int64_t>(row) * H + c * 8, o);
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[p] = dot;
  }
  grid_done_signal(counter, target, P.flags, 3 * kEPMax + P.rank, P.world, seq);
}

// Backward of the dispatch: dx[t] = sum_s dx_owner[dest_row[t,s]] (P2P pulls).
// Waits for channel 4.
__global__ void ep_dispatch_bwd_kernel(EPPeers P, const int* __restrict__ idx, const int* __restrict__ dest_row,
                                       __nv_bfloat16* __restrict__ dx, int N, int K, int H, int El,
                                       unsigned seq, int* err) {
  if (!block_wait_flags(P.flags[P.rank] + 4 * kEPMax, P.world, seq, err)) return;
  const int H8 = H / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < static_cast<int64_t>(N) * H8;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int t = static_cast<int>(v / H8);
    const int c = static_cast<int>(v - static_cast<int64_t>(t) * H8);
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int s = 0; s < K; ++s) {
      const int64_t p = static_cast<int64_t>(t) * K + s;
      const int row = dest_row[p];
      if (row < 0) continue;
      const int d = idx[p] / El;
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(P.buf[d] + static_cast<int64_t>(row) * H) + c);
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(hv[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    store8(dx + static_cast<int64_t>(t) * H + c * 8, acc);
  }
}

// --------------------------------------------------------------------- host
static int ep_grid(int64_t work, int threads) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + threads - 1) / threads, num_sms() * 8)));
}

void ep_layout(std::vector<int64_t> flags, std::vector<int64_t> counts, int64_t rank, torch::Tensor counts_local,
               int64_t E, int64_t El, int64_t seq, torch::Tensor dest_base, torch::Tensor seg_off,
               torch::Tensor seg_used, int64_t cap) {
  TORCH_CHECK(E <= kEPMaxE && E % El == 0, "ep_layout: experts");
  auto P = make_ep(flags, counts, {}, rank);
  TORCH_CHECK(E == El * P.world, "ep_layout: E = El * world");
  auto st = at::cuda::getCurrentCUDAStream();
  ep_layout_kernel<<<1, 256, 0, st>>>(P, counts_local.data_ptr<float>(), static_cast<int>(E), static_cast<int>(El),
                                      static_cast<unsigned>(seq), dest_base.data_ptr<int>(), seg_off.data_ptr<int>(),
                                      seg_used.data_ptr<int>(), static_cast<int>(cap), error_flag_ptr());
  NQ_CHECK_CUDA(cudaGetLastError());
}

int64_t ep_dispatch(std::vector<int64_t> flags, std::vector<int64_t> counts, std::vector<int64_t> recv, int64_t rank,
                    torch::Tensor x, torch::Tensor idx, torch::Tensor slot_of, torch::Tensor loc_off,
                    torch::Tensor dest_base, torch::Tensor seg_off, torch::Tensor seg_used, torch::Tensor dest_row,
                    int64_t El, int64_t cap, int64_t seq, torch::Tensor counter, int64_t counter_before) {
  auto P = make_ep(flags, counts, recv, rank);
  check_bf16(x, "x");
  const int N = x.size(0), H = x.size(1), K = idx.size(1);
  TORCH_CHECK(H % 8 == 0, "ep_dispatch: hidden % 8");
  const int grid = ep_grid(static_cast<int64_t>(N) * K * 32, 256);
  auto st = at::cuda::getCurrentCUDAStream();
  ep_dispatch_kernel<<<grid, 256, 0, st>>>(
      P, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), idx.data_ptr<int>(), slot_of.data_ptr<int>(),
      loc_off.data_ptr<int>(), dest_base.data_ptr<int>(), seg_off.data_ptr<int>(), seg_used.data_ptr<int>(),
      dest_row.data_ptr<int>(), N, K, H, static_cast<int>(El), static_cast<int>(cap), static_cast<unsigned>(seq),
      reinterpret_cast<unsigned*>(counter.data_ptr()), static_cast<unsigned>(counter_before + grid), error_flag_ptr());
  NQ_CHECK_CUDA(cudaGetLastError());
  return grid;
}

void ep_wait(std::vector<int64_t> flags, std::vector<int64_t> counts, int64_t rank, int64_t ch, int64_t seq) {
  auto P = make_ep(flags, counts, {}, rank);
  ep_wait_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(P, static_cast<int>(ch), static_cast<unsigned>(seq),
                                                                  error_flag_ptr());
  NQ_CHECK_CUDA(cudaGetLastError());
}

void ep_signal(std::vector<int64_t> flags, std::vector<int64_t> counts, int64_t rank, int64_t ch, int64_t seq) {
  auto P = make_ep(flags, counts, {}, rank);
  ep_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(P, static_cast<int>(ch), static_cast<unsigned>(seq));
  NQ_CHECK_CUDA(cudaGetLastError());
}

void ep_combine(std::vector<int64_t> flags, std::vector<int64_t> counts, std::vector<int64_t> yout, int64_t rank,
                torch::Tensor idx, torch::Tensor dest_row, torch::Tensor w, torch::Tensor out, torch::Tensor y_pulled,
                int64_t El, int64_t seq) {
  auto P = make_ep(flags, counts, yout, rank);
  const int N = out.size(0), H = out.size(1), K = idx.size(1);
  const int grid = ep_grid(static_cast<int64_t>(N) * (H / 8), 256);
  ep_combine_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      P, idx.data_ptr<int>(), dest_row.data_ptr<int>(), w.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y_pulled.data_ptr()), N, K,
      H, static_cast<int>(El), static_cast<unsigned>(seq), error_flag_ptr());
  NQ_CHECK_CUDA(cudaGetLastError());
}

int64_t ep_combine_bwd(std::vector<int64_t> flags, std::vector<int64_t> counts, std::vector<int64_t> dyrecv,
                       int64_t rank, torch::Tensor idx, torch::Tensor dest_row, torch::Tensor w, torch::Tensor dout,
                       torch::Tensor y_pulled, torch::Tensor dw, int64_t El, int64_t seq, torch::Tensor counter,
                       int64_t counter_before) {
  auto P = make_ep(flags, counts, dyrecv, rank);
  const int N = dout.size(0), H = dout.size(1), K = idx.size(1);
  const int grid = ep_grid(static_cast<int64_t>(N) * K * 32, 256);
  ep_combine_bwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      P, idx.data_ptr<int>(), dest_row.data_ptr<int>(), w.data_ptr<float>(),
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(y_pulled.data_ptr()),
      dw.data_ptr<float>(), N, K, H, static_cast<int>(El), static_cast<unsigned>(seq),
      reinterpret_cast<unsigned*>(counter.data_ptr()), static_cast<unsigned>(counter_before + grid));
  NQ_CHECK_CUDA(cudaGetLastError());
  return grid;
}

void ep_dispatch_bwd(std::vector<int64_t> flags, std::vector<int64_t> counts, std::vector<int64_t> dxrecv, int64_t rank,
                     torch::Tensor idx, torch::Tensor dest_row, torch::Tensor dx, int64_t El, int64_t seq) {
  auto P = make_ep(flags, counts, dxrecv, rank);
  const int N = dx.size(0), H = dx.size(1), K = idx.size(1);
  const int grid = ep_grid(static_cast<int64_t>(N) * (H / 8), 256);
  ep_dispatch_bwd_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      P, idx.data_ptr<int>(), dest_row.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), N, K, H,
      static_cast<int>(El), static_cast<unsigned>(seq), error_flag_ptr());
  NQ_CHECK_CUDA(cudaGetLastError());
}

}  // namespace nq
