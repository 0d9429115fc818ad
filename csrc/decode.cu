// KV-cache attention for generation (decode and short prefill chunks).
//
// Split-K "flash decoding": CTA = (batch, kv-head, key split).  The CTA loads
// the queries of every q-head of the GQA group once, streams its share of the
// cache in 128-key chunks (one key per thread for the scores, one head-dim
// column per thread for P V), keeps an online softmax per query row, and
// writes a partial (O, max, sum).  A second kernel merges the splits.  The
// split count depends only on the cache capacity, so shapes are static and the
// step can be captured in a CUDA graph; valid lengths are read on the device.
// Causality: query row i (absolute position q_start+i) sees keys <= q_start+i.
#include "common.cuh"
#include "tmap.h"

namespace nq {

constexpr int kDecThreads = 128;
constexpr int kDecChunk = 128;
constexpr int kDecMaxRows = 32;  // (q-heads per kv head) * query rows

template <int D>
__global__ void __launch_bounds__(kDecThreads) decode_partial_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
    const __nv_bfloat16* __restrict__ vc, const int* __restrict__ cache_len,
    const int* __restrict__ q_start, float* __restrict__ part_o, float* __restrict__ part_m,
    float* __restrict__ part_l, int Sq, int Hq, int Hk, int Smax, int splits, float scale_log2) {
  const int split = blockIdx.x % splits;
  const int bh = blockIdx.x / splits;
  const int b = bh / Hk;
  const int hk = bh - b * Hk;
  const int G = Hq / Hk;
  const int nrows = G * Sq;  // row = g * Sq + i
  __shared__ float sq[kDecMaxRows][D];
  __shared__ float sp[kDecMaxRows][kDecChunk];
  __shared__ float sm[kDecMaxRows], sl[kDecMaxRows], salpha[kDecMaxRows];
  const int tid = threadIdx.x;
  for (int e = tid; e < nrows * D; e += blockDim.x) {
    const int row = e / D, d = e - row * D;
    const int g = row / Sq, i = row - g * Sq;
    sq[row][d] = __bfloat162float(q[((static_cast<int64_t>(b) * Sq + i) * Hq + hk * G + g) * D + d]);
  }
  if (tid < nrows) { sm[tid] = -INFINITY; sl[tid] = 0.f; }
  float acc[kDecMaxRows];
#pragma unroll
  for (int r = 0; r < kDecMaxRows; ++r) acc[r] = 0.f;
  __syncthreads();
  const int len = cache_len[b];
  const int qs = q_start[b];
  const int per = (Smax + splits - 1) / splits;
  const int kb = split * per;
  const int ke = min(min(kb + per, Smax), len);
  for (int c0 = kb; c0 < ke; c0 += kDecChunk) {
    // scores: thread = key
    const int kj = c0 + tid;
    if (kj < ke) {
      const __nv_bfloat16* kr = kc + ((static_cast<int64_t>(b) * Smax + kj) * Hk + hk) * D;
      float kv[D];
#pragma unroll
      for (int d = 0; d < D; d += 8) {
        float f[8];
        load8(kr + d, f);
#pragma unroll
        for (int i = 0; i < 8; ++i) kv[d + i] = f[i];
      }
      for (int row = 0; row < nrows; ++row) {
        const int i = row % Sq;
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) s += sq[row][d] * kv[d];
        sp[row][tid] = (kj <= qs + i) ? s * scale_log2 : -INFINITY;
      }
    } else {
      for (int row = 0; row < nrows; ++row) sp[row][tid] = -INFINITY;
    }
    __syncthreads();
    // online softmax per row: one warp per row
    const int warp = tid >> 5, lane = tid & 31;
    for (int row = warp; row < nrows; row += blockDim.x / 32) {
      float mx = -INFINITY;
      for (int j = lane; j < kDecChunk; j += 32) mx = fmaxf(mx, sp[row][j]);
      mx = warp_max(mx);
      const float mo = sm[row];
      const float mn = fmaxf(mo, mx);
      float sum = 0.f;
      for (int j = lane; j < kDecChunk; j += 32) {
        const float p = (mn == -INFINITY) ? 0.f : exp2f(sp[row][j] - mn);
        sp[row][j] = p;
        sum += p;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float a = (mo == -INFINITY) ? 0.f : exp2f(mo - mn);
        salpha[row] = a;
        sl[row] = sl[row] * a + sum;
        sm[row] = mn;
      }
    }
    __syncthreads();
    // P V: thread = head-dim column
    if (tid < D) {
      for (int row = 0; row < nrows; ++row) acc[row] *= salpha[row];
      const int n = min(kDecChunk, ke - c0);
      for (int j = 0; j < n; ++j) {
        const float v = __bfloat162float(vc[((static_cast<int64_t>(b) * Smax + c0 + j) * Hk + hk) * D + tid]);
#pragma unroll 4
        for (int row = 0; row < nrows; ++row) acc[row] += sp[row][j] * v;
      }
    }
    __syncthreads();
  }
  // write partials
  for (int row = 0; row < nrows; ++row) {
    const int g = row / Sq, i = row - g * Sq;
    const int64_t pidx = ((static_cast<int64_t>(b) * Hq + hk * G + g) * Sq + i) * splits + split;
    if (tid < D) part_o[pidx * D + tid] = acc[row];
    if (tid == 0) { part_m[pidx] = sm[row]; part_l[pidx] = sl[row]; }
  }
}

template <int D>
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_m,
                                      const float* __restrict__ part_l, __nv_bfloat16* __restrict__ out,
                                      int rows, int splits, int Sq, int Hq) {
  const int row = blockIdx.x;  // (b, h, i)
  if (row >= rows) return;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, part_m[static_cast<int64_t>(row) * splits + s]);
  float l = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = part_m[static_cast<int64_t>(row) * splits + s];
    if (m != -INFINITY) l += part_l[static_cast<int64_t>(row) * splits + s] * exp2f(m - mx);
  }
  const int i = row % Sq;
  const int bh = row / Sq;
  const int h = bh % Hq;
  const int b = bh / Hq;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float m = part_m[static_cast<int64_t>(row) * splits + s];
      if (m != -INFINITY) o += part_o[(static_cast<int64_t>(row) * splits + s) * D + d] * exp2f(m - mx);
    }
    out[((static_cast<int64_t>(b) * Sq + i) * Hq + h) * D + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
  }
}

// q [B, Sq, Hq, D]; caches [B, Smax, Hk, D] (token-major, contiguous); returns [B, Sq, Hq, D].
torch::Tensor decode_attn(torch::Tensor q, torch::Tensor kc, torch::Tensor vc, torch::Tensor cache_len,
                          torch::Tensor q_start, double scale) {
  check_bf16(q, "q"); check_bf16(kc, "k_cache"); check_bf16(vc, "v_cache");
  TORCH_CHECK(kc.is_contiguous() && vc.is_contiguous(), "decode_attn: caches contiguous");
  auto qc = q.contiguous();
  const int B = qc.size(0), Sq = qc.size(1), Hq = qc.size(2), D = qc.size(3);
  const int Smax = kc.size(1), Hk = kc.size(2);
  TORCH_CHECK((Hq / Hk) * Sq <= kDecMaxRows, "decode_attn: (Hq/Hk)*Sq must be <= 32 (use the prefill kernel)");
  c10::cuda::CUDAGuard g(q.device());
  auto cl = cache_len.to(torch::kInt32).contiguous();
  auto qs = q_start.to(torch::kInt32).contiguous();
  const int want = std::max(1, (2 * num_sms() + B * Hk - 1) / (B * Hk));
  const int splits = std::max(1, std::min(want, (Smax + 255) / 256));
  auto opt = q.options().dtype(torch::kFloat32);
  const int64_t rows = static_cast<int64_t>(B) * Hq * Sq;
  auto po = torch::empty({rows * splits, D}, opt);
  auto pm = torch::empty({rows * splits}, opt);
  auto pl = torch::empty({rows * splits}, opt);
  auto out = torch::empty_like(qc);
  auto st = at::cuda::getCurrentCUDAStream();
  const float sl2 = static_cast<float>(scale) * 1.4426950408889634f;
  if (D == 128) {
    decode_partial_kernel<128><<<B * Hk * splits, kDecThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(qc.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr()), cl.data_ptr<int>(), qs.data_ptr<int>(),
        po.data_ptr<float>(), pm.data_ptr<float>(), pl.data_ptr<float>(), Sq, Hq, Hk, Smax, splits, sl2);
    decode_combine_kernel<128><<<rows, 128, 0, st>>>(po.data_ptr<float>(), pm.data_ptr<float>(), pl.data_ptr<float>(),
                                                     reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, splits, Sq, Hq);
  } else if (D == 64) {
    decode_partial_kernel<64><<<B * Hk * splits, kDecThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(qc.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr()), cl.data_ptr<int>(), qs.data_ptr<int>(),
        po.data_ptr<float>(), pm.data_ptr<float>(), pl.data_ptr<float>(), Sq, Hq, Hk, Smax, splits, sl2);
    decode_combine_kernel<64><<<rows, 64, 0, st>>>(po.data_ptr<float>(), pm.data_ptr<float>(), pl.data_ptr<float>(),
                                                   reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, splits, Sq, Hq);
  } else {
    TORCH_CHECK(false, "decode_attn: head_dim 64 or 128");
  }
  NQ_CHECK_CUDA(cudaGetLastError());
  return out;
}

}  // namespace nq


// ----------------------------------------------------------------------------
// Allocation-free entry point (declared, with its contract, in
// decode_noalloc.h).  Same kernels and split choice as decode_attn above; the
// split-K partials go to a fixed file-scope device array instead of buffers
// from PyTorch's allocator.
#include <mutex>
#include <cstdio>
#include "decode_noalloc.h"

namespace nq {
namespace {

constexpr size_t kNoAllocScratchFloats = NQ_DECODE_NOALLOC_SCRATCH_BYTES / sizeof(float);
// Host code sees this name only as a symbol handle; its device address comes
// from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_decode_scratch[kNoAllocScratchFloats];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};

int noalloc_fail(char* err, int err_len, int code, const char* msg) {
  if (err != nullptr && err_len > 0) std::snprintf(err, static_cast<size_t>(err_len), "%s", msg);
  return code;
}

}  // namespace
}  // namespace nq

extern "C" int nq_decode_attn_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                      const int* cache_len, const int* q_start, void* out, int B,
                                      int Sq, int Hq, int Hk, int D, int Smax, float scale,
                                      cudaStream_t stream, char* err, int err_len) {
  using namespace nq;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || cache_len == nullptr ||
      q_start == nullptr || out == nullptr)
    return noalloc_fail(err, err_len, NQ_NOALLOC_BAD_ARG, "nq_decode_attn_noalloc: null pointer");
  if (B <= 0 || Sq <= 0 || Hq <= 0 || Hk <= 0 || Smax <= 0 || Hq % Hk != 0)
    return noalloc_fail(err, err_len, NQ_NOALLOC_BAD_ARG,
                        "nq_decode_attn_noalloc: bad shape (B, Sq, Hq, Hk, Smax > 0; Hq % Hk == 0)");
  if (D != 64 && D != 128)
    return noalloc_fail(err, err_len, NQ_NOALLOC_BAD_ARG, "nq_decode_attn_noalloc: head_dim must be 64 or 128");
  if ((Hq / Hk) * Sq > kDecMaxRows)
    return noalloc_fail(err, err_len, NQ_NOALLOC_BAD_ARG,
                        "nq_decode_attn_noalloc: (Hq/Hk)*Sq must be <= 32");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
    return noalloc_fail(err, err_len, NQ_NOALLOC_CUDA_ERROR, "nq_decode_attn_noalloc: cudaGetDevice failed");
  const int want = std::max(1, (2 * num_sms() + B * Hk - 1) / (B * Hk));
  const int splits = std::max(1, std::min(want, (Smax + 255) / 256));
  const size_t rows = static_cast<size_t>(B) * Hq * Sq;
  const size_t need = rows * splits * (static_cast<size_t>(D) + 2);
  if (need > kNoAllocScratchFloats) {
    char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "nq_decode_attn_noalloc: needs %zu bytes of scratch, the library's fixed maximum is %zu bytes "
                  "(reduce batch, heads, query rows or cache length)",
                  need * sizeof(float), static_cast<size_t>(NQ_DECODE_NOALLOC_SCRATCH_BYTES));
    return noalloc_fail(err, err_len, NQ_NOALLOC_TOO_LARGE, msg);
  }
  float* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* p = nullptr;
      const cudaError_t rc = cudaGetSymbolAddress(&p, g_decode_scratch);
      if (rc != cudaSuccess || p == nullptr) {
        char msg[256];
        std::snprintf(msg, sizeof(msg), "nq_decode_attn_noalloc: cudaGetSymbolAddress failed: %s",
                      cudaGetErrorString(rc));
        return noalloc_fail(err, err_len, NQ_NOALLOC_CUDA_ERROR, msg);
      }
      g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    base = g_noalloc_ptr[dev];
  }
  float* po = base;
  float* pm = po + rows * splits * D;
  float* pl = pm + rows * splits;
  const float sl2 = scale * 1.4426950408889634f;
  const auto* qb = static_cast<const __nv_bfloat16*>(q);
  const auto* kb = static_cast<const __nv_bfloat16*>(k_cache);
  const auto* vb = static_cast<const __nv_bfloat16*>(v_cache);
  auto* ob = static_cast<__nv_bfloat16*>(out);
  if (D == 128) {
    decode_partial_kernel<128><<<B * Hk * splits, kDecThreads, 0, stream>>>(
        qb, kb, vb, cache_len, q_start, po, pm, pl, Sq, Hq, Hk, Smax, splits, sl2);
    decode_combine_kernel<128><<<static_cast<int>(rows), 128, 0, stream>>>(po, pm, pl, ob, static_cast<int>(rows),
                                                                        splits, Sq, Hq);
  } else {
    decode_partial_kernel<64><<<B * Hk * splits, kDecThreads, 0, stream>>>(
        qb, kb, vb, cache_len, q_start, po, pm, pl, Sq, Hq, Hk, Smax, splits, sl2);
    decode_combine_kernel<64><<<static_cast<int>(rows), 64, 0, stream>>>(po, pm, pl, ob, static_cast<int>(rows),
                                                                      splits, Sq, Hq);
  }
  const cudaError_t rc = cudaGetLastError();
  if (rc != cudaSuccess) {
    char msg[256];
    std::snprintf(msg, sizeof(msg), "nq_decode_attn_noalloc: launch failed: %s", cudaGetErrorString(rc));
    return noalloc_fail(err, err_len, NQ_NOALLOC_CUDA_ERROR, msg);
  }
  return NQ_NOALLOC_OK;
}
