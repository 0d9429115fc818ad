// Tensor/sequence-parallel communication fused into the residual-add +
// RMSNorm kernels (forward and backward) over NVLink peer memory.
//
// Under sequence parallelism each rank holds R = T / tp rows of the residual
// stream.  Around every column-parallel GEMM (q|k|v, gate|up) the normalised
// rows must be all-gathered, and every row-parallel GEMM (o_proj, down_proj)
// produces a partial sum over the full sequence that must be reduce-scattered.
// Here:
//
//  * the row-parallel GEMM's epilogue stores each finished row tile straight
//    into the owning rank's partial buffer `parts[src]` (csrc/gemm.cu, RS
//    epilogue) and the GEMM's last CTA publishes a flag;
//  * tp_norm_fwd_kernel waits (bounded) for every source's flag, sums the tp
//    partials into the residual (the reduce-scatter's reduction), normalises,
//    and stores the bf16 row into every rank's full-sequence buffer (the
//    all-gather) before its last CTA publishes the all-gather flag;
//  * the column-parallel GEMM's TMA producer waits for the owner's flag before
//    loading an A tile of the full buffer (csrc/gemm.cu, AG wait).
//
// The backward kernel mirrors this: it sums the reduce-scattered partials of
// d(normalised input) written by the column-parallel dgrad GEMMs, and
// all-gathers the bf16 residual gradient that the row-parallel GEMMs consume.
// Flags follow peer.cuh (monotonic sequence numbers, bounded waits).  Flag
// block per rank: [4 channels][8 sources] u32; channel 0 = all-gather fwd,
// 1 = reduce-scatter fwd, 2 = all-gather bwd, 3 = reduce-scatter bwd.
#include "common.cuh"
#include "peer.cuh"
#include "tmap.h"

namespace nq {

constexpr int kTPMax = 8;
constexpr int kTPThreads = 256;

struct TPSync {
  unsigned* flags_local;          // this rank's flag block
  unsigned* flags_peer[kTPMax];   // every rank's flag block (mapped)
  int world, rank;
  int wait_ch;                    // channel to wait on before reading partials (-1: none)
  unsigned wait_seq;
  int sig_ch;                     // channel to publish after the all-gather stores (-1: none)
  unsigned sig_seq;
  unsigned* counter;              // local monotonic block counter
  unsigned target;                // counter value after this launch
  int* err;
};

template <typename T> __device__ __forceinline__ void tld8(const T* p, float (&f)[8]) { load8(p, f); }
template <typename T> __device__ __forceinline__ void tst8(T* p, const float (&f)[8]) { store8(p, f); }

// h = resid (+ delta) (+ sum_s parts[s]); y = bf16(h * rstd * w) -> local y and
// every ag_dst[r] (+ row offset).
template <int NCH>
__global__ void __launch_bounds__(kTPThreads) tp_norm_fwd_kernel(
    const float* __restrict__ resid, const __nv_bfloat16* __restrict__ delta,
    const __nv_bfloat16* __restrict__ parts, const float* __restrict__ w, float* __restrict__ h_out,
    __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, TPSync S,
    int R, int H, float eps,
    __nv_bfloat16* ag0, __nv_bfloat16* ag1, __nv_bfloat16* ag2, __nv_bfloat16* ag3,
    __nv_bfloat16* ag4, __nv_bfloat16* ag5, __nv_bfloat16* ag6, __nv_bfloat16* ag7) {
  __nv_bfloat16* ag[kTPMax] = {ag0, ag1, ag2, ag3, ag4, ag5, ag6, ag7};
  __shared__ float red[32];
  if (S.wait_ch >= 0 && parts != nullptr) {
    if (!block_wait_flags(S.flags_local + S.wait_ch * kTPMax, S.world, S.wait_seq, S.err)) return;
  }
  const int64_t plane = static_cast<int64_t>(R) * H;
  for (int row = blockIdx.x; row < R; row += gridDim.x) {
    float v[NCH][8];
    float ss = 0.f;
    const int64_t base = static_cast<int64_t>(row) * H;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kTPThreads + threadIdx.x) * 8;
      if (col < H) {
        tld8(resid + base + col, v[c]);
        if (delta != nullptr) {
          float d[8];
          tld8(delta + base + col, d);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[c][i] += d[i];
        }
        if (parts != nullptr) {
          for (int s = 0; s < S.world; ++s) {
            float d[8];
            tld8(parts + s * plane + base + col, d);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[c][i] += d[i];
          }
        }
        tst8(h_out + base + col, v[c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
      }
    }
    ss = block_sum(ss, red);
    const float r = rsqrtf(ss / H + eps);
    if (threadIdx.x == 0) rstd_out[row] = r;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kTPThreads + threadIdx.x) * 8;
      if (col < H) {
        float wv[8], o[8];
        tld8(w + col, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[c][i] * r * wv[i];
        tst8(y + base + col, o);
#pragma unroll
        for (int q = 0; q < kTPMax; ++q)
          if (q < S.world && ag[q] != nullptr) tst8(ag[q] + base + col, o);
      }
    }
  }
  if (S.sig_ch >= 0)
    grid_done_signal(S.counter, S.target, S.flags_peer, S.sig_ch * kTPMax + S.rank, S.world, S.sig_seq);
}

// Backward of h = resid + delta, y = h * rstd * w, with dy either local or the
// sum of tp partials; dx (fp32) = dh + rstd * (g - xhat * mean(g * xhat)),
// g = dy * w.  The bf16 copy of dx goes to local dx_bf16 and every ag[r].
template <int NCH>
__global__ void __launch_bounds__(kTPThreads) tp_norm_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ dy_parts,
    const float* __restrict__ dh, const float* __restrict__ h, const float* __restrict__ w,
    const float* __restrict__ rstd, float* __restrict__ dx, __nv_bfloat16* __restrict__ dx_bf16,
    float* __restrict__ dw_part, TPSync S, int R, int H,
    __nv_bfloat16* ag0, __nv_bfloat16* ag1, __nv_bfloat16* ag2, __nv_bfloat16* ag3,
    __nv_bfloat16* ag4, __nv_bfloat16* ag5, __nv_bfloat16* ag6, __nv_bfloat16* ag7) {
  __nv_bfloat16* ag[kTPMax] = {ag0, ag1, ag2, ag3, ag4, ag5, ag6, ag7};
  __shared__ float red[32];
  if (S.wait_ch >= 0 && dy_parts != nullptr) {
    if (!block_wait_flags(S.flags_local + S.wait_ch * kTPMax, S.world, S.wait_seq, S.err)) return;
  }
  const int64_t plane = static_cast<int64_t>(R) * H;
  float dwacc[NCH][8], wv[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * kTPThreads + threadIdx.x) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) dwacc[c][i] = 0.f;
    if (col < H) tld8(w + col, wv[c]);
  }
  for (int row = blockIdx.x; row < R; row += gridDim.x) {
    const int64_t base = static_cast<int64_t>(row) * H;
    const float r = rstd[row];
    float xh[NCH][8], g[NCH][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kTPThreads + threadIdx.x) * 8;
      if (col < H) {
        float hv[8], d[8];
        tld8(h + base + col, hv);
        if (dy != nullptr) {
          tld8(dy + base + col, d);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) d[i] = 0.f;
        }
        if (dy_parts != nullptr) {
          for (int s = 0; s < S.world; ++s) {
            float e[8];
            tld8(dy_parts + s * plane + base + col, e);
#pragma unroll
            for (int i = 0; i < 8; ++i) d[i] += e[i];
          }
        }
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
      const int col = (c * kTPThreads + threadIdx.x) * 8;
      if (col < H) {
        float o[8], res[8];
        if (dh != nullptr) tld8(dh + base + col, res);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = r * (g[c][i] - xh[c][i] * dot) + (dh != nullptr ? res[i] : 0.f);
        tst8(dx + base + col, o);
        tst8(dx_bf16 + base + col, o);
#pragma unroll
        for (int q = 0; q < kTPMax; ++q)
          if (q < S.world && ag[q] != nullptr) tst8(ag[q] + base + col, o);
      }
    }
  }
  if (dw_part != nullptr) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = (c * kTPThreads + threadIdx.x) * 8;
      if (col < H) tst8(dw_part + static_cast<int64_t>(blockIdx.x) * H + col, dwacc[c]);
    }
  }
  if (S.sig_ch >= 0)
    grid_done_signal(S.counter, S.target, S.flags_peer, S.sig_ch * kTPMax + S.rank, S.world, S.sig_seq);
}

__global__ void tp_colsum_add_kernel(const float* __restrict__ part, int G, int H, float* __restrict__ out) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= H) return;
  float s = 0.f;
  for (int b = 0; b < G; ++b) s += part[static_cast<int64_t>(b) * H + col];
  out[col] += s;
}

// ---------------------------------------------------------------------- host
static TPSync make_sync(torch::Tensor flags_local, const std::vector<int64_t>& flags_peer, int64_t rank,
                        int64_t wait_ch, int64_t wait_seq, int64_t sig_ch, int64_t sig_seq,
                        torch::Tensor counter, int64_t target) {
  TPSync S{};
  S.world = static_cast<int>(flags_peer.size());
  TORCH_CHECK(S.world >= 1 && S.world <= kTPMax, "tp: 1..8 ranks");
  S.rank = static_cast<int>(rank);
  S.flags_local = reinterpret_cast<unsigned*>(flags_local.data_ptr());
  for (int r = 0; r < S.world; ++r) S.flags_peer[r] = reinterpret_cast<unsigned*>(flags_peer[r]);
  S.wait_ch = static_cast<int>(wait_ch);
  S.wait_seq = static_cast<unsigned>(wait_seq);
  S.sig_ch = static_cast<int>(sig_ch);
  S.sig_seq = static_cast<unsigned>(sig_seq);
  S.counter = reinterpret_cast<unsigned*>(counter.data_ptr());
  S.target = static_cast<unsigned>(target);
  S.err = error_flag_ptr();
  return S;
}

static int tp_grid(int R) { return std::max(1, std::min(R, num_sms() * 8)); }

static void ag_ptrs(const std::vector<int64_t>& ag, __nv_bfloat16* (&out)[kTPMax]) {
  TORCH_CHECK(ag.size() <= static_cast<size_t>(kTPMax), "tp: at most 8 all-gather targets");
  for (int i = 0; i < kTPMax; ++i)
    out[i] = i < static_cast<int>(ag.size()) ? reinterpret_cast<__nv_bfloat16*>(ag[i]) : nullptr;
}

// Returns the grid size the caller must add to the block counter.
int64_t tp_norm_fwd(torch::Tensor resid, c10::optional<torch::Tensor> delta, c10::optional<torch::Tensor> parts,
                    torch::Tensor w, torch::Tensor h_out, torch::Tensor y, torch::Tensor rstd, double eps,
                    std::vector<int64_t> ag, torch::Tensor flags_local, std::vector<int64_t> flags_peer,
                    int64_t rank, int64_t wait_ch, int64_t wait_seq, int64_t sig_ch, int64_t sig_seq,
                    torch::Tensor counter, int64_t counter_before) {
  const int R = resid.size(0), H = resid.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * kTPThreads * 4, "tp_norm_fwd: hidden size");
  const int grid = tp_grid(R);
  auto S = make_sync(flags_local, flags_peer, rank, wait_ch, wait_seq, sig_ch, sig_seq, counter,
                     counter_before + grid);
  __nv_bfloat16* a[kTPMax];
  ag_ptrs(ag, a);
  const __nv_bfloat16* dp = (delta.has_value() && delta->defined())
                                ? reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr()) : nullptr;
  const __nv_bfloat16* pp = (parts.has_value() && parts->defined())
                                ? reinterpret_cast<const __nv_bfloat16*>(parts->data_ptr()) : nullptr;
  auto st = at::cuda::getCurrentCUDAStream();
  const int nch = (H / 8 + kTPThreads - 1) / kTPThreads;
#define NQ_TPN_LAUNCH(N)                                                                            \
  tp_norm_fwd_kernel<N><<<grid, kTPThreads, 0, st>>>(                                               \
      resid.data_ptr<float>(), dp, pp, w.data_ptr<float>(), h_out.data_ptr<float>(),                \
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), S, R, H,              \
      static_cast<float>(eps), a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7])
  if (nch <= 1) NQ_TPN_LAUNCH(1);
  else if (nch <= 2) NQ_TPN_LAUNCH(2);
  else NQ_TPN_LAUNCH(4);
#undef NQ_TPN_LAUNCH
  NQ_CHECK_CUDA(cudaGetLastError());
  return grid;
}

int64_t tp_norm_bwd(c10::optional<torch::Tensor> dy, c10::optional<torch::Tensor> dy_parts,
                    c10::optional<torch::Tensor> dh, torch::Tensor h, torch::Tensor w, torch::Tensor rstd,
                    torch::Tensor dx, torch::Tensor dx_bf16, c10::optional<torch::Tensor> dw,
                    std::vector<int64_t> ag, torch::Tensor flags_local, std::vector<int64_t> flags_peer,
                    int64_t rank, int64_t wait_ch, int64_t wait_seq, int64_t sig_ch, int64_t sig_seq,
                    torch::Tensor counter, int64_t counter_before) {
  const int R = h.size(0), H = h.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * kTPThreads * 4, "tp_norm_bwd: hidden size");
  const int grid = tp_grid(R);
  auto S = make_sync(flags_local, flags_peer, rank, wait_ch, wait_seq, sig_ch, sig_seq, counter,
                     counter_before + grid);
  __nv_bfloat16* a[kTPMax];
  ag_ptrs(ag, a);
  auto opt_bf = [](const c10::optional<torch::Tensor>& t) -> const __nv_bfloat16* {
    return (t.has_value() && t->defined()) ? reinterpret_cast<const __nv_bfloat16*>(t->data_ptr()) : nullptr;
  };
  const float* dhp = (dh.has_value() && dh->defined()) ? dh->data_ptr<float>() : nullptr;
  torch::Tensor part;
  float* dwp = nullptr;
  if (dw.has_value() && dw->defined()) {
    part = torch::empty({grid, H}, h.options());
    dwp = part.data_ptr<float>();
  }
  auto st = at::cuda::getCurrentCUDAStream();
  const int nch = (H / 8 + kTPThreads - 1) / kTPThreads;
#define NQ_TPB_LAUNCH(N)                                                                            \
  tp_norm_bwd_kernel<N><<<grid, kTPThreads, 0, st>>>(                                               \
      opt_bf(dy), opt_bf(dy_parts), dhp, h.data_ptr<float>(), w.data_ptr<float>(), rstd.data_ptr<float>(), \
      dx.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dx_bf16.data_ptr()), dwp, S, R, H,    \
      a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7])
  if (nch <= 1) NQ_TPB_LAUNCH(1);
  else if (nch <= 2) NQ_TPB_LAUNCH(2);
  else NQ_TPB_LAUNCH(4);
#undef NQ_TPB_LAUNCH
  NQ_CHECK_CUDA(cudaGetLastError());
  if (dwp != nullptr) {
    tp_colsum_add_kernel<<<(H + 255) / 256, 256, 0, st>>>(dwp, grid, H, dw->data_ptr<float>());
    NQ_CHECK_CUDA(cudaGetLastError());
  }
  return grid;
}

}  // namespace nq
