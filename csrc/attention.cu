// Causal / non-causal GQA flash attention for sm_100a (tcgen05 + TMEM + TMA).
//
// Layout: q|k rows [T, (Hq+Hk)*D] and v inside the packed q|k|v rows
// [T, (Hq+2Hk)*D] (T = B*S, token-major), so no head transposes exist anywhere.
// GQA is native: q head h reads kv head h / (Hq/Hk).
//
// Forward CTA (one (batch, q-head, 128-query block)), 6 warps:
//   warp 0   : TMA producer: Q once, then K_j / V_j into a 2-stage ring;
//   warp 1   : MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM
//              S buffers, O += P_{j-1} V_{j-1} into the TMEM O accumulator,
//              software-pipelined so softmax(j) overlaps P V (j-1);
//   warps 2-5: softmax warpgroup, thread = query row = TMEM lane: reads S_j,
//              masks, exponentiates (exp2 domain), writes bf16 P into a 128B-
//              swizzled SMEM tile (the A operand of P V), and rescales O in
//              TMEM only when the running max grows by more than 2^8 (exact:
//              the final O / l uses the same reference max).
// Output: bf16 O [T, Hq*D] and fp32 log-sum-exp [B, Hq, S].
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace nq {

constexpr int ABM = 128;      // queries per CTA
constexpr int ABN = 128;      // keys per block
constexpr int kAttnThreads = 192;
constexpr int kKVStages = 2;
constexpr float kRescaleThresh = 8.0f;  // log2 units

template <int D>
struct AttnFwdSmem {
  static constexpr int kQBytes = ABM * D * 2;
  static constexpr int kKBytes = ABN * D * 2;
  static constexpr int kVBytes = ABN * D * 2;
  static constexpr int kPBytes = ABM * ABN * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + kKVStages * kKBytes;
  static constexpr int kPOff = kVOff + kKVStages * kVBytes;
  static constexpr int kBarOff = kPOff + kPBytes;
  static constexpr int kBytes = kBarOff + 256 + 1024;
};

struct AttnArgs {
  int B, S, Hq, Hk;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  __nv_bfloat16* O;  // [T, Hq*D]
  float* lse;        // [B, Hq, S]
  int* err;
};

// Write one row of 128 bf16 values (given as fp32) into a K-major SW128 tile
// made of 64-column regions of ABM rows (region stride ABM*128 bytes).
__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int row, int col0, const float* v,
                                                int nrows_region) {
  // col0 is a multiple of 8; writes 8 values (one 16-byte unit)
  const int region = col0 >> 6;
  const int unit = (col0 & 63) >> 3;
  uint8_t* base = tile + region * nrows_region * 128 + row * 128 + ((unit ^ (row & 7)) << 4);
  uint4 u;
  u.x = pack_bf16(v[0], v[1]);
  u.y = pack_bf16(v[2], v[3]);
  u.z = pack_bf16(v[4], v[5]);
  u.w = pack_bf16(v[6], v[7]);
  *reinterpret_cast<uint4*>(base) = u;
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQK, const __grid_constant__ CUtensorMap tmV,
                    const AttnArgs args) {
  using L = AttnFwdSmem<D>;
  constexpr int KCH = D / 64;  // 64-wide d chunks
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint8_t* sP = smem + L::kPOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* v_full = bars + 3;   // [2]
  uint64_t* kv_empty = bars + 5; // [2]
  uint64_t* s_full = bars + 7;   // [2]
  uint64_t* s_free = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = args.err;

  const int S = args.S;
  const int n_mblk = (S + ABM - 1) / ABM;
  // Heaviest (last) query blocks first for causal load balance.
  const int mb = n_mblk - 1 - (blockIdx.x % n_mblk);
  const int bh = blockIdx.x / n_mblk;
  const int b = bh / args.Hq;
  const int h = bh - b * args.Hq;
  const int hk = h / (args.Hq / args.Hk);
  const int q0 = mb * ABM;               // first query (within the sequence)
  const int tok0 = b * S;                // first token of the sequence
  const int n_kblk = args.causal ? min((q0 + ABM + ABN - 1) / ABN, (S + ABN - 1) / ABN)
                                 : (S + ABN - 1) / ABN;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;          // two S buffers: cols [0,128), [128,256)
  const uint32_t tO = tmem + 256;    // O accumulator: cols [256, 256+D)

  if (warp == 0) {
    if (elect_one()) {
      bool ok = true;
      mbar_arrive_expect_tx(q_full, L::kQBytes);
#pragma unroll
      for (int c = 0; c < KCH; ++c) tma_load_3d(sQ + c * ABM * 128, &tmQK, q_full, c * 64, h, tok0 + q0);
      for (int j = 0; j < n_kblk && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, err, kErrTimeoutProducer)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[st], L::kKBytes);
#pragma unroll
        for (int c = 0; c < KCH; ++c)
          tma_load_3d(sK + st * L::kKBytes + c * ABN * 128, &tmQK, &k_full[st], c * 64, args.Hq + hk, tok0 + j * ABN);
        mbar_arrive_expect_tx(&v_full[st], L::kVBytes);
#pragma unroll
        for (int c = 0; c < KCH; ++c)
          tma_load_3d(sV + st * L::kVBytes + c * ABN * 128, &tmV, &v_full[st], c * 64, args.Hq + args.Hk + hk, tok0 + j * ABN);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_bf16(ABM, ABN, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16(ABM, D, false, true);
      bool ok = mbar_wait(q_full, 0, err, kErrTimeoutMma);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_pv = [&](int jj) -> bool {
        const int st = jj & 1;
        if (!mbar_wait(p_full, jj & 1, err, kErrTimeoutMma)) return false;
        if (!mbar_wait(&v_full[st], (jj >> 1) & 1, err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP);
        const uint32_t v_addr = smem_u32(sV + st * L::kVBytes);
#pragma unroll
        for (int kk = 0; kk < ABN / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(p_addr + (kk >> 2) * (ABM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(v_addr + kk * 2048, ABN * 128, 1024);
          umma_bf16(tO, ad, bd, idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&kv_empty[st]);
        return true;
      };
      for (int j = 0; j < n_kblk && ok; ++j) {
        const int st = j & 1;
        const int sb = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, err, kErrTimeoutMma)) { ok = false; break; }
        if (!mbar_wait(&s_free[sb], ((j >> 1) & 1) ^ 1, err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * L::kKBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(q_addr + (kk >> 2) * (ABM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_addr + (kk >> 2) * (ABN * 128) + (kk & 3) * 32, 16, 1024);
          umma_bf16(tS + sb * ABN, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) issue_pv(n_kblk - 1);
    }
  } else {
    // -------------------------------------------------------- softmax WG
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row within the tile == TMEM lane
    const int qi = q0 + r;              // query position within the sequence
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float m_ref = -INFINITY;  // reference max (log2 domain, scaled)
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kblk; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1, err, kErrTimeoutSoftmax)) { ok = false; break; }
      tc_fence_after();
      float s[ABN];
#pragma unroll
      for (int c = 0; c < ABN; c += 32) {
        uint32_t u[32];
        tmem_ld32(tS + lane_base + sb * ABN + c, u);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c + i] = __uint_as_float(u[i]) * args.scale_log2;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sb]);
      const int k0 = j * ABN;
      const bool need_mask = (args.causal && k0 + ABN - 1 > q0) || (k0 + ABN > S);
      float mx = -INFINITY;
      if (need_mask) {
#pragma unroll
        for (int i = 0; i < ABN; ++i) {
          const int kj = k0 + i;
          if (kj >= S || (args.causal && kj > qi)) s[i] = -INFINITY;
          mx = fmaxf(mx, s[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < ABN; ++i) mx = fmaxf(mx, s[i]);
      }
      // Lazy rescale: move the reference max only when it grew by > 2^8.
      const bool grow = mx > m_ref + kRescaleThresh;
      const float m_new = grow ? mx : m_ref;
      const float alpha = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - m_new);
      float rowsum = 0.f;
      const bool dead = (m_new == -INFINITY);
#pragma unroll
      for (int i = 0; i < ABN; ++i) {
        s[i] = dead ? 0.f : exp2f(s[i] - m_new);
        rowsum += s[i];
      }
      // P buffer and O are busy until the previous P V completes.
      if (j > 0) {
        if (!mbar_wait(pv_done, (j - 1) & 1, err, kErrTimeoutSoftmax)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow && m_ref != -INFINITY)) {
          const float a = grow ? alpha : 1.f;
#pragma unroll
          for (int c = 0; c < D; c += 16) {
            uint32_t u[16];
            tmem_ld16(tO + lane_base + c, u);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * a);
            tmem_st16(tO + lane_base + c, u);
          }
          tmem_wait_st();
        }
      }
      l = l * (grow ? alpha : 1.f) + rowsum;
      m_ref = m_new;
#pragma unroll
      for (int c = 0; c < ABN; c += 8) store_row_sw128(sP, r, c, &s[c], ABM);
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // --------------------------------------------------------- epilogue
    if (ok && mbar_wait(pv_done, (n_kblk - 1) & 1, err, kErrTimeoutSoftmax)) {
      tc_fence_after();
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      const bool row_ok = qi < S;
      __nv_bfloat16* orow = args.O + (static_cast<int64_t>(tok0 + qi) * args.Hq + h) * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t u[32];
        tmem_ld32(tO + lane_base + c, u);
        tmem_wait_ld();
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(u[q * 8 + 0]) * inv_l, __uint_as_float(u[q * 8 + 1]) * inv_l);
            v.y = pack_bf16(__uint_as_float(u[q * 8 + 2]) * inv_l, __uint_as_float(u[q * 8 + 3]) * inv_l);
            v.z = pack_bf16(__uint_as_float(u[q * 8 + 4]) * inv_l, __uint_as_float(u[q * 8 + 5]) * inv_l);
            v.w = pack_bf16(__uint_as_float(u[q * 8 + 6]) * inv_l, __uint_as_float(u[q * 8 + 7]) * inv_l);
            dst[q] = v;
          }
        }
      }
      if (row_ok) {
        const float lse = (l > 0.f) ? (m_ref + __log2f(l)) * 0.6931471805599453f : -INFINITY;
        args.lse[(static_cast<int64_t>(b) * args.Hq + h) * S + qi] = lse;
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

// --------------------------------------------------------------------- host
template <int D>
static void launch_attn_fwd(const torch::Tensor& qk, const torch::Tensor& qkv, torch::Tensor& o,
                            torch::Tensor& lse, int B, int S, int Hq, int Hk, bool causal, float scale) {
  using L = AttnFwdSmem<D>;
  const int64_t T = static_cast<int64_t>(B) * S;
  auto tq = make_tmap_3d_bf16(qk.data_ptr(), D, Hq + Hk, T, D, (int64_t)(Hq + Hk) * D, 64, 1, ABM);
  auto tv = make_tmap_3d_bf16(qkv.data_ptr(), D, Hq + 2 * Hk, T, D, (int64_t)(Hq + 2 * Hk) * D, 64, 1, ABN);
  AttnArgs a;
  a.B = B; a.S = S; a.Hq = Hq; a.Hk = Hk;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal = causal ? 1 : 0;
  a.O = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.err = error_flag_ptr();
  auto kern = attn_fwd_kernel<D>;
  static bool attr = false;
  if (!attr) {
    NQ_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes));
    attr = true;
  }
  const int grid = B * Hq * ((S + ABM - 1) / ABM);
  kern<<<grid, kAttnThreads, L::kBytes, at::cuda::getCurrentCUDAStream()>>>(tq, tv, a);
  NQ_CHECK_CUDA(cudaGetLastError());
}

std::vector<torch::Tensor> attn_fwd(torch::Tensor qk, torch::Tensor qkv, int64_t B, int64_t S,
                                    int64_t Hq, int64_t Hk, int64_t D, bool causal, double scale) {
  check_bf16(qk, "qk"); check_bf16(qkv, "qkv");
  TORCH_CHECK(qk.is_contiguous() && qkv.is_contiguous(), "attn_fwd: contiguous inputs");
  TORCH_CHECK(qk.size(1) == (Hq + Hk) * D && qkv.size(1) == (Hq + 2 * Hk) * D, "attn_fwd: widths");
  TORCH_CHECK(Hq % Hk == 0, "attn_fwd: Hq % Hk");
  c10::cuda::CUDAGuard g(qk.device());
  auto o = torch::empty({B * S, Hq * D}, qk.options());
  auto lse = torch::empty({B, Hq, S}, qk.options().dtype(torch::kFloat32));
  if (B * S == 0) return {o, lse};
  if (D == 128) launch_attn_fwd<128>(qk, qkv, o, lse, B, S, Hq, Hk, causal, (float)scale);
  else if (D == 64) launch_attn_fwd<64>(qk, qkv, o, lse, B, S, Hq, Hk, causal, (float)scale);
  else TORCH_CHECK(false, "attn_fwd: head_dim must be 64 or 128");
  return {o, lse};
}

}  // namespace nq
