// Flash-attention backward for sm_100a (tcgen05 + TMEM + TMA).
//
// CTA = (batch, kv-head, 128-key block).  K and V stay resident in shared
// memory; the CTA walks every q-head of its GQA group and every query block
// that can see its keys (causal), and for each one issues five tcgen05 GEMMs:
//   S^T  = K Q^T,  dP^T = V dO^T          (TMEM; thread = key row)
//   P^T  = exp(S^T * scale - lse),  dS^T = P^T (dP^T - delta) * scale  (bf16 -> SMEM)
//   dV  += P^T dO,  dK += dS^T Q          (TMEM accumulators for the whole walk)
//   dQ_i = dS K                           (TMEM, then vector atomics into fp32 dQ)
// The dS^T tile written K-major for dK is read MN-major as the A operand of dQ
// (same 128B-swizzled bytes), so no transpose pass exists.  delta = rowsum(dO*O)
// comes from a small pre-pass kernel that also zeroes the dQ accumulator.
// Outputs: dq|dk fp32 [T, (Hq+Hk)*D]; dv bf16 written into the v slot of dqkv.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace nq {

constexpr int BKN = 128;  // keys per CTA
constexpr int BQM = 128;  // queries per iteration
constexpr int kBwdThreads = 192;

template <int D>
struct AttnBwdSmem {
  static constexpr int kTile = 128 * D * 2;  // K, V, Q, dO tiles
  static constexpr int kPT = BKN * BQM * 2;
  static constexpr int kKOff = 0;
  static constexpr int kVOff = kKOff + kTile;
  static constexpr int kQOff = kVOff + kTile;
  static constexpr int kDOOff = kQOff + kTile;
  static constexpr int kPTOff = kDOOff + kTile;
  static constexpr int kDSOff = kPTOff + kPT;
  static constexpr int kLseOff = kDSOff + kPT;          // 128 floats lse (log2 domain), 128 delta
  static constexpr int kBarOff = kLseOff + 2 * BQM * 4;
  static constexpr int kBytes = kBarOff + 256 + 1024;
};

struct AttnBwdArgs {
  int B, S, Hq, Hk;
  float scale;        // softmax scale
  float scale_log2;   // scale * log2(e)
  int causal;
  const float* lse;   // [B, Hq, S] natural log
  const float* delta; // [B, Hq, S]
  float* dqk;         // [T, (Hq+Hk)*D] fp32: dq accumulated by atomics, dk written
  __nv_bfloat16* dqkv;  // [T, (Hq+2Hk)*D]: dv written into the v slot
  int* err;
};

__device__ __forceinline__ void store8_sw128(uint8_t* tile, int row, int col0, const float* v) {
  const int region = col0 >> 6;
  const int unit = (col0 & 63) >> 3;
  uint8_t* p = tile + region * (128 * 128) + row * 128 + ((unit ^ (row & 7)) << 4);
  uint4 u;
  u.x = pack_bf16(v[0], v[1]);
  u.y = pack_bf16(v[2], v[3]);
  u.z = pack_bf16(v[4], v[5]);
  u.w = pack_bf16(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ void wg_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQK, const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmDO, const AttnBwdArgs args) {
  using L = AttnBwdSmem<D>;
  constexpr int KCH = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sDO = smem + L::kDOOff;
  uint8_t* sPT = smem + L::kPTOff;
  uint8_t* sDS = smem + L::kDSOff;
  float* sLse = reinterpret_cast<float*>(smem + L::kLseOff);
  float* sDelta = sLse + BQM;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;
  uint64_t* qdo_empty = bars + 2;
  uint64_t* s_full = bars + 3;    // S^T and dP^T ready
  uint64_t* pt_full = bars + 4;   // P^T / dS^T written (and S^T/dP^T consumed)
  uint64_t* pt_free = bars + 5;   // MMAs reading P^T / dS^T done
  uint64_t* dq_full = bars + 6;
  uint64_t* st_free = bars + 7;   // dQ read out of TMEM
  uint64_t* acc_done = bars + 8;  // final dK / dV
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = args.err;
  const int S = args.S;
  const int n_kblk = (S + BKN - 1) / BKN;
  const int nb = blockIdx.x % n_kblk;
  const int bk = blockIdx.x / n_kblk;
  const int b = bk / args.Hk;
  const int hk = bk - b * args.Hk;
  const int G = args.Hq / args.Hk;
  const int k0 = nb * BKN;
  const int tok0 = b * S;
  const int n_mblk = (S + BQM - 1) / BQM;
  const int mb_begin = args.causal ? (k0 / BQM) : 0;
  const int iters_per_head = n_mblk - mb_begin;
  const int n_iter = G * iters_per_head;

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(&bars[i], (i == 4 || i == 7) ? 4u : 1u);  // pt_full, st_free: 4 warps
    fence_barrier_init();
    tma_prefetch_desc(&tmQK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tST = tmem;         // S^T, later dQ
  const uint32_t tDP = tmem + 128;   // dP^T
  const uint32_t tDK = tmem + 256;
  const uint32_t tDV = tmem + 384;

  auto iter_coords = [&](int it, int& hq, int& mb) {
    const int g = it / iters_per_head;
    hq = hk * G + g;
    mb = mb_begin + (it - g * iters_per_head);
  };

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * L::kTile);
#pragma unroll
      for (int c = 0; c < KCH; ++c) {
        tma_load_3d(sK + c * 128 * 128, &tmQK, kv_full, c * 64, args.Hq + hk, tok0 + k0);
        tma_load_3d(sV + c * 128 * 128, &tmV, kv_full, c * 64, args.Hq + args.Hk + hk, tok0 + k0);
      }
      for (int it = 0; it < n_iter; ++it) {
        int hq, mb;
        iter_coords(it, hq, mb);
        if (!mbar_wait(qdo_empty, (it & 1) ^ 1, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(qdo_full, 2 * L::kTile);
#pragma unroll
        for (int c = 0; c < KCH; ++c) {
          tma_load_3d(sQ + c * 128 * 128, &tmQK, qdo_full, c * 64, hq, tok0 + mb * BQM);
          tma_load_3d(sDO + c * 128 * 128, &tmDO, qdo_full, c * 64, hq, tok0 + mb * BQM);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t id_s = idesc_bf16(BKN, BQM, false, false);   // K Q^T, V dO^T
      constexpr uint32_t id_kv = idesc_bf16(BKN, D, false, true);     // P^T dO, dS^T Q
      constexpr uint32_t id_q = idesc_bf16(BQM, D, true, true);       // dS K
      bool ok = mbar_wait(kv_full, 0, err, kErrTimeoutMma);
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aQ = smem_u32(sQ), aDO = smem_u32(sDO);
      const uint32_t aPT = smem_u32(sPT), aDS = smem_u32(sDS);
      for (int it = 0; it < n_iter && ok; ++it) {
        const uint32_t ph = it & 1;
        if (!mbar_wait(qdo_full, ph, err, kErrTimeoutMma)) { ok = false; break; }
        if (!mbar_wait(st_free, ph ^ 1, err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          umma_bf16(tST, sdesc_sw128(aK + off, 16, 1024), sdesc_sw128(aQ + off, 16, 1024), id_s, kk > 0);
          umma_bf16(tDP, sdesc_sw128(aV + off, 16, 1024), sdesc_sw128(aDO + off, 16, 1024), id_s, kk > 0);
        }
        umma_commit(s_full);
        if (!mbar_wait(pt_full, ph, err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        // dV += P^T dO ; dK += dS^T Q   (K = queries)
#pragma unroll
        for (int kk = 0; kk < BQM / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          const uint32_t boff = kk * 2048;
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          umma_bf16(tDV, sdesc_sw128(aPT + aoff, 16, 1024), sdesc_sw128(aDO + boff, 128 * 128, 1024), id_kv, acc);
          umma_bf16(tDK, sdesc_sw128(aDS + aoff, 16, 1024), sdesc_sw128(aQ + boff, 128 * 128, 1024), id_kv, acc);
        }
        // dQ = dS K   (M = queries, K = keys): A = dS^T tile read MN-major, B = K read MN-major
#pragma unroll
        for (int kk = 0; kk < BKN / 16; ++kk) {
          umma_bf16(tST, sdesc_sw128(aDS + kk * 2048, 128 * 128, 1024),
                    sdesc_sw128(aK + kk * 2048, 128 * 128, 1024), id_q, kk > 0);
        }
        umma_commit(dq_full);
        umma_commit(qdo_empty);
        umma_commit(pt_free);
      }
      if (ok) umma_commit(acc_done);
    }
  } else {
    // ------------------------------------------------------- compute WG
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int tid = threadIdx.x - 64;  // 0..127
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int kj = k0 + r;             // this thread's key position
    bool ok = true;
    for (int it = 0; it < n_iter; ++it) {
      int hq, mb;
      iter_coords(it, hq, mb);
      const uint32_t ph = it & 1;
      const int q0 = mb * BQM;
      // per-query lse (log2 domain) and delta into shared memory
      {
        const int q = q0 + tid;
        const int64_t idx = (static_cast<int64_t>(b) * args.Hq + hq) * S + q;
        sLse[tid] = (q < S) ? args.lse[idx] * 1.4426950408889634f : INFINITY;
        sDelta[tid] = (q < S) ? args.delta[idx] : 0.f;
      }
      wg_sync();
      if (!mbar_wait(s_full, ph, err, kErrTimeoutSoftmax)) { ok = false; break; }
      tc_fence_after();
      // previous iteration's MMAs must be done reading sPT / sDS
      if (!mbar_wait(pt_free, ph ^ 1, err, kErrTimeoutSoftmax)) { ok = false; break; }
#pragma unroll 1
      for (int c = 0; c < BQM; c += 32) {
        uint32_t us[32], ud[32];
        tmem_ld32(tST + lane_base + c, us);
        tmem_ld32(tDP + lane_base + c, ud);
        tmem_wait_ld();
        float p[32], ds[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int qi = q0 + c + i;
          const bool masked = (qi >= S) || (kj >= S) || (args.causal && kj > qi);
          const float pv = masked ? 0.f : exp2f(__uint_as_float(us[i]) * args.scale_log2 - sLse[c + i]);
          p[i] = pv;
          ds[i] = pv * (__uint_as_float(ud[i]) - sDelta[c + i]) * args.scale;
        }
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          store8_sw128(sPT, r, c + i, &p[i]);
          store8_sw128(sDS, r, c + i, &ds[i]);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pt_full);
      // dQ tile (thread = query row r) -> atomics into fp32 dq
      if (!mbar_wait(dq_full, ph, err, kErrTimeoutSoftmax)) { ok = false; break; }
      tc_fence_after();
      const int qrow = q0 + r;
      float* dq = args.dqk + (static_cast<int64_t>(tok0 + qrow) * (args.Hq + args.Hk) + hq) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t u[32];
        tmem_ld32(tST + lane_base + c, u);
        tmem_wait_ld();
        if (qrow < S) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            atomicAdd(reinterpret_cast<float4*>(dq + c + i),
                      make_float4(__uint_as_float(u[i]), __uint_as_float(u[i + 1]),
                                  __uint_as_float(u[i + 2]), __uint_as_float(u[i + 3])));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(st_free);
    }
    // ------------------------------------------------------- dK / dV out
    if (ok && n_iter > 0 && mbar_wait(acc_done, 0, err, kErrTimeoutSoftmax)) {
      tc_fence_after();
      const bool row_ok = kj < S;
      float* dk = args.dqk + (static_cast<int64_t>(tok0 + kj) * (args.Hq + args.Hk) + args.Hq + hk) * D;
      __nv_bfloat16* dv = args.dqkv + (static_cast<int64_t>(tok0 + kj) * (args.Hq + 2 * args.Hk) + args.Hq + args.Hk + hk) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t uk[32], uv[32];
        tmem_ld32(tDK + lane_base + c, uk);
        tmem_ld32(tDV + lane_base + c, uv);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dk + c + i) = make_float4(__uint_as_float(uk[i]), __uint_as_float(uk[i + 1]),
                                                               __uint_as_float(uk[i + 2]), __uint_as_float(uk[i + 3]));
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(uv[q * 8 + 0]), __uint_as_float(uv[q * 8 + 1]));
            v.y = pack_bf16(__uint_as_float(uv[q * 8 + 2]), __uint_as_float(uv[q * 8 + 3]));
            v.z = pack_bf16(__uint_as_float(uv[q * 8 + 4]), __uint_as_float(uv[q * 8 + 5]));
            v.w = pack_bf16(__uint_as_float(uv[q * 8 + 6]), __uint_as_float(uv[q * 8 + 7]));
            reinterpret_cast<uint4*>(dv + c)[q] = v;
          }
        }
      }
    } else if (n_iter == 0) {
      // no query can see these keys: zero gradients
      if (kj < S) {
        float* dk = args.dqk + (static_cast<int64_t>(tok0 + kj) * (args.Hq + args.Hk) + args.Hq + hk) * D;
        __nv_bfloat16* dv = args.dqkv + (static_cast<int64_t>(tok0 + kj) * (args.Hq + 2 * args.Hk) + args.Hq + args.Hk + hk) * D;
        for (int c = 0; c < D; ++c) { dk[c] = 0.f; dv[c] = __float2bfloat16_rn(0.f); }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[b,h,q] = sum_d dO * O ; also zeroes the dq part of dqk.
template <int D>
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* __restrict__ dO, const __nv_bfloat16* __restrict__ O,
                                    float* __restrict__ delta, float* __restrict__ dqk, int B, int S,
                                    int Hq, int Hk) {
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t items = static_cast<int64_t>(B) * S * Hq;
  for (int64_t it = gw; it < items; it += warps) {
    const int64_t t = it / Hq;
    const int h = static_cast<int>(it - t * Hq);
    const __nv_bfloat16* a = dO + (t * Hq + h) * D;
    const __nv_bfloat16* o = O + (t * Hq + h) * D;
    float s = 0.f;
    for (int d = lane * 2; d < D; d += 64) {
      const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(a + d));
      const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(o + d));
      s += x.x * y.x + x.y * y.y;
    }
    s = warp_sum(s);
    const int b = static_cast<int>(t / S);
    const int q = static_cast<int>(t - static_cast<int64_t>(b) * S);
    if (lane == 0) delta[(static_cast<int64_t>(b) * Hq + h) * S + q] = s;
    float* dq = dqk + (t * (Hq + Hk) + h) * D;
    for (int d = lane * 4; d < D; d += 128) *reinterpret_cast<float4*>(dq + d) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <int D>
static torch::Tensor launch_attn_bwd(const torch::Tensor& dO, const torch::Tensor& qk, const torch::Tensor& qkv,
                                     const torch::Tensor& O, const torch::Tensor& lse, torch::Tensor& dqkv,
                                     int B, int S, int Hq, int Hk, bool causal, float scale) {
  using L = AttnBwdSmem<D>;
  const int64_t T = static_cast<int64_t>(B) * S;
  auto dqk = torch::empty({T, (int64_t)(Hq + Hk) * D}, qk.options().dtype(torch::kFloat32));
  auto delta = torch::empty({B, Hq, S}, qk.options().dtype(torch::kFloat32));
  auto st = at::cuda::getCurrentCUDAStream();
  {
    const int64_t items = T * Hq;
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((items + 7) / 8, num_sms() * 8)));
    attn_bwd_pre_kernel<D><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(dO.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(O.data_ptr()),
        delta.data_ptr<float>(), dqk.data_ptr<float>(), B, S, Hq, Hk);
    NQ_CHECK_CUDA(cudaGetLastError());
  }
  auto tq = make_tmap_3d_bf16(qk.data_ptr(), D, Hq + Hk, T, D, (int64_t)(Hq + Hk) * D, 64, 1, 128);
  auto tv = make_tmap_3d_bf16(qkv.data_ptr(), D, Hq + 2 * Hk, T, D, (int64_t)(Hq + 2 * Hk) * D, 64, 1, 128);
  auto tdo = make_tmap_3d_bf16(dO.data_ptr(), D, Hq, T, D, (int64_t)Hq * D, 64, 1, 128);
  AttnBwdArgs a;
  a.B = B; a.S = S; a.Hq = Hq; a.Hk = Hk;
  a.scale = scale;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal = causal ? 1 : 0;
  a.lse = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.dqk = dqk.data_ptr<float>();
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.err = error_flag_ptr();
  auto kern = attn_bwd_kernel<D>;
  static bool attr = false;
  if (!attr) {
    NQ_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    attr = true;
  }
  const int grid = B * Hk * ((S + BKN - 1) / BKN);
  kern<<<grid, kBwdThreads, L::kBytes, st>>>(tq, tv, tdo, a);
  NQ_CHECK_CUDA(cudaGetLastError());
  return dqk;
}

// Returns dq|dk fp32 [T, (Hq+Hk)*D]; writes dv (bf16) into the v slot of dqkv.
torch::Tensor attn_bwd(torch::Tensor dO, torch::Tensor qk, torch::Tensor qkv, torch::Tensor O,
                       torch::Tensor lse, torch::Tensor dqkv, int64_t B, int64_t S, int64_t Hq,
                       int64_t Hk, int64_t D, bool causal, double scale) {
  check_bf16(dO, "dO"); check_bf16(qk, "qk"); check_bf16(qkv, "qkv"); check_bf16(O, "O"); check_bf16(dqkv, "dqkv");
  TORCH_CHECK(dO.is_contiguous() && O.is_contiguous() && dqkv.is_contiguous(), "attn_bwd: contiguous");
  c10::cuda::CUDAGuard g(qk.device());
  if (D == 128) return launch_attn_bwd<128>(dO, qk, qkv, O, lse, dqkv, B, S, Hq, Hk, causal, (float)scale);
  if (D == 64) return launch_attn_bwd<64>(dO, qk, qkv, O, lse, dqkv, B, S, Hq, Hk, causal, (float)scale);
  TORCH_CHECK(false, "attn_bwd: head_dim must be 64 or 128");
  return torch::Tensor();
}

}  // namespace nq
