// Causal / non-causal GQA flash attention forward for sm_100a
// (tcgen05 + TMEM + TMA).
//
// Layout: q|k rows [T, (Hq+Hk)*D] and v inside the packed q|k|v rows
// [T, (Hq+2Hk)*D] (T = B*S, token-major), so no head transposes exist anywhere.
// GQA is native: q head h reads kv head h / (Hq/Hk).
//
// CTA = (batch, q-head, 256 queries) = two 128-row query tiles, 12 warps:
//   warp 0     : TMA producer: Q0/Q1 once, then 64-key K_j / V_j tiles into a
//                4-stage ring;
//   warp 1     : MMA issuer (one thread).  S_t(j) = Q_t K_j^T goes to buffer
//                j % 2 of tile t; once tile t's softmax published P_t(j) it
//                issues O_t += P_t(j) V(j) (A operand P read from TMEM) and
//                then S_t(j+2) into the buffer P_t(j) occupied, so S_t(j+1)
//                is already in TMEM when the softmax finishes block j and the
//                tensor core alternates between the two tiles;
//   warps 4-7  : softmax warpgroup for tile 0, warps 8-11 for tile 1; thread =
//                query row = TMEM lane.  Reads S (fp32), masks, exponentiates
//                in the exp2 domain with tree reductions, writes P as packed
//                bf16 back into TMEM over S, and rescales O in TMEM only when
//                the running max grew by more than 2^8 (exact: the final O / l
//                uses the same reference max).
// TMEM: tile t's two S/P buffers at cols [128t, 128t+64) and [128t+64,
// 128t+128) (64 keys each; P packed bf16 in a buffer's first 32 columns),
// O tile 0 [256,256+D), O tile 1 [384,384+D).  Outputs bf16 O [T, Hq*D] and fp32 LSE [B, Hq, S].
#include "common.cuh"
#include "peer.cuh"
#include "tmap.h"

namespace nq {

constexpr int ABM = 128;        // queries per tile
constexpr int ABN = 64;         // keys per block
constexpr int NKV = 4;          // K/V ring stages
constexpr int kTilesPerCta = 2;
constexpr int kAttnThreads = 384;
constexpr float kRescaleThresh = 8.0f;  // log2 units

template <int D>
struct AttnFwdSmem {
  static constexpr int kQBytes = ABM * D * 2;   // per tile
  static constexpr int kKVBytes = ABN * D * 2;  // K or V per stage
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kTilesPerCta * kQBytes;
  static constexpr int kVOff = kKOff + NKV * kKVBytes;
  static constexpr int kBarOff = kVOff + NKV * kKVBytes;
  static constexpr int kBytes = kBarOff + 256 + 1024;
};

struct AttnArgs {
  int B, S, Hq, Hk;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  __nv_bfloat16* O;  // [T, Hq*D]
  float* lse;        // [B, Hq, S]
  int* err;
  // Keys/values: rows per batch (Sk), head index of K and V in their tensor
  // maps.  Queries: key-space position of query row i is i + off0 for
  // i < split, else i + off1 (context parallelism: a rank's two zigzag chunks
  // against the gathered keys).  Self-attention: Sk = S, offsets 0.
  int Sk, k_head, v_head, off0, off1, split;
  // Peer-memory K/V gather (context parallelism): before loading the key block
  // at position p, wait until kv_flags[owner(p)] reaches kv_seq, where
  // owner(p) = zigzag owner of chunk p / cp_c among cp_world ranks.  null: no wait.
  const unsigned* kv_flags;
  unsigned kv_seq;
  int cp_c, cp_world;
  // Key-range mask (document packing, left padding): query token i sees keys
  // [kv_lo[i], i] of its row; kv_lo is non-decreasing along a row.  The CTA
  // skips every key block before kv_lo of its first query.  null: causal only.
  const int* kv_lo;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32"
      " [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Hardware 2^x (MUFU), relative error ~2^-22; ample for bf16 probabilities.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQK, const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmK, const AttnArgs args) {
  using L = AttnFwdSmem<D>;
  constexpr int KCH = D / 64;  // 64-wide d chunks
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [NKV]
  uint64_t* v_full = bars + 5;    // [NKV]
  uint64_t* kv_empty = bars + 9;  // [NKV]
  uint64_t* s_full = bars + 13;   // [tile * 2 + buffer]
  uint64_t* p_full = bars + 17;   // [2] per tile (P written, S consumed)
  uint64_t* o_done = bars + 19;   // [2] per tile: PV(j) complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 23);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = args.err;

  const int S = args.S;
  constexpr int CTA_M = ABM * kTilesPerCta;
  const int n_mblk = (S + CTA_M - 1) / CTA_M;
  // Heaviness-major order: the first wave holds the longest causal tiles of
  // every (batch, head), the lightest run last (longest-processing-time-first
  // scheduling by the hardware block scheduler); adjacent blocks are adjacent
  // heads, which share K/V under GQA.
  const int n_bh = gridDim.x / n_mblk;
  const int mb = n_mblk - 1 - static_cast<int>(blockIdx.x) / n_bh;
  const int bh = static_cast<int>(blockIdx.x) % n_bh;
  const int b = bh / args.Hq;
  const int h = bh - b * args.Hq;
  const int hk = h / (args.Hq / args.Hk);
  const int q0 = mb * CTA_M;
  const int tok0 = b * S;
  const int Sk = args.Sk;
  const int ktok0 = b * Sk;
  const int qoff = (q0 < args.split) ? args.off0 : args.off1;  // CTA rows share one chunk
  const int n_kend = args.causal ? min((q0 + qoff + CTA_M + ABN - 1) / ABN, (Sk + ABN - 1) / ABN)
                                 : (Sk + ABN - 1) / ABN;
  // first key block (key-range mask); the loops below count iterations j from
  // 0 and read key block jb + j
  const int jb = (args.kv_lo != nullptr) ? min(args.kv_lo[tok0 + q0] / ABN, n_kend) : 0;
  const int n_kblk = n_kend - jb;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NKV; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&p_full[s], 4);
      mbar_init(&o_done[s], 1);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmQK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmK);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      bool ok = true;
      mbar_arrive_expect_tx(q_full, kTilesPerCta * L::kQBytes);
#pragma unroll
      for (int t = 0; t < kTilesPerCta; ++t)
#pragma unroll
        for (int c = 0; c < KCH; ++c)
          tma_load_3d(sQ + t * L::kQBytes + c * ABM * 128, &tmQK, q_full, c * 64, h, tok0 + q0 + t * ABM);
      int waited = -1;
      for (int j = 0; j < n_kblk && ok; ++j) {
        const int st = j % NKV;
        const uint32_t ph = static_cast<uint32_t>(j / NKV) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, err, kErrTimeoutProducer)) { ok = false; break; }
        if (args.kv_flags != nullptr) {
          const int chunk = ((jb + j) * ABN) / args.cp_c;
          const int owner = chunk < args.cp_world ? chunk : 2 * args.cp_world - 1 - chunk;
          if (owner != waited) {
            if (!wait_flag(args.kv_flags + owner, args.kv_seq, err)) { ok = false; break; }
            asm volatile("fence.proxy.async.global;" ::: "memory");
            waited = owner;
          }
        }
        mbar_arrive_expect_tx(&k_full[st], L::kKVBytes);
#pragma unroll
        for (int c = 0; c < KCH; ++c)
          tma_load_3d(sK + st * L::kKVBytes + c * ABN * 128, &tmK, &k_full[st], c * 64, args.k_head + hk, ktok0 + (jb + j) * ABN);
        mbar_arrive_expect_tx(&v_full[st], L::kKVBytes);
#pragma unroll
        for (int c = 0; c < KCH; ++c)
          tma_load_3d(sV + st * L::kKVBytes + c * ABN * 128, &tmV, &v_full[st], c * 64, args.v_head + hk, ktok0 + (jb + j) * ABN);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_bf16(ABM, ABN, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16(ABM, D, false, true);
      bool ok = mbar_wait(q_full, 0, err, kErrTimeoutMma);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ);
      // S_t(j) into buffer j % 2 of tile t (after P_t(j-2) was consumed by
      // PV_t(j-2), issued earlier on this thread: MMAs execute in order).
      auto issue_qk = [&](int j, int t) -> bool {
        const int st = j % NKV;
        if (!mbar_wait(&k_full[st], static_cast<uint32_t>(j / NKV) & 1, err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t tS = tmem + t * 128 + (j & 1) * ABN;
        const uint32_t k_addr = smem_u32(sK + st * L::kKVBytes);
        const uint32_t qa = q_addr + t * L::kQBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(qa + (kk >> 2) * (ABM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_addr + (kk >> 2) * (ABN * 128) + (kk & 3) * 32, 16, 1024);
          umma_bf16(tS, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t * 2 + (j & 1)]);
        return true;
      };
      for (int j = 0; j < min(2, n_kblk) && ok; ++j) {
        for (int t = 0; t < kTilesPerCta && ok; ++t) ok = issue_qk(j, t);
      }
      for (int j = 0; j < n_kblk && ok; ++j) {
        const int st = j % NKV;
        if (!mbar_wait(&v_full[st], static_cast<uint32_t>(j / NKV) & 1, err, kErrTimeoutMma)) { ok = false; break; }
        const uint32_t v_addr = smem_u32(sV + st * L::kKVBytes);
#pragma unroll
        for (int t = 0; t < kTilesPerCta; ++t) {
          const uint32_t tP = tmem + t * 128 + (j & 1) * ABN;
          const uint32_t tO = tmem + 256 + t * 128;
          // P_t(j) is ready once its softmax finished
          if (!mbar_wait(&p_full[t], j & 1, err, kErrTimeoutMma)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < ABN / 16; ++kk) {
            const uint64_t bd = sdesc_sw128(v_addr + kk * 2048, ABN * 128, 1024);
            umma_bf16_ts(tO, tP + kk * 8, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&o_done[t]);
          if (j + 2 < n_kblk && !issue_qk(j + 2, t)) { ok = false; break; }
        }
        if (!ok) break;
        umma_commit(&kv_empty[st]);  // K(j) and V(j) no longer read
      }
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------- softmax WGs
    const int t = (warp - 4) >> 2;          // tile
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;      // row in tile == TMEM lane
    const int qi = q0 + t * ABM + r;        // query position in the sequence
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tO = tmem + 256 + t * 128 + lane_base;
    float m_ref = -INFINITY;
    float l = 0.f;
    bool ok = true;
    const int lo = (args.kv_lo != nullptr) ? args.kv_lo[tok0 + min(qi, S - 1)] : 0;
    for (int j = 0; j < n_kblk; ++j) {
      if (!mbar_wait(&s_full[t * 2 + (j & 1)], static_cast<uint32_t>(j >> 1) & 1, err, kErrTimeoutSoftmax)) {
        ok = false;
        break;
      }
      const uint32_t tS = tmem + t * 128 + (j & 1) * ABN + lane_base;
      tc_fence_after();
      // The two tiles exponentiate independently: with S double-buffered, a
      // tile whose next S is ready starts at once (forcing the two tiles'
      // exponential phases to alternate measured 10% slower).
      constexpr int NCK = ABN / 32;  // 32-column chunks of a block
      uint32_t u[NCK][32];
#pragma unroll
      for (int c = 0; c < NCK; ++c) tmem_ld32(tS + c * 32, u[c]);
      tmem_wait_ld();
      const int k0 = (jb + j) * ABN;
      const bool need_mask = (args.causal && k0 + ABN - 1 > q0 + qoff + t * ABM) || (k0 + ABN > Sk) ||
                             (k0 < lo);
      // Raw scores stay in registers; the scale (> 0) is applied to the max and
      // folded into the exponent's FFMA.
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < NCK; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int kj = k0 + c * 32 + i;
            if (kj >= Sk || (args.causal && kj > qi + qoff) || kj < lo) u[c][i] = 0xff800000u;  // -inf
          }
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < NCK; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], __uint_as_float(u[c][i]));
      const float sl2 = args.scale_log2;
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
      const bool grow = mx > m_ref + kRescaleThresh;
      const float m_new = grow ? mx : m_ref;
      const bool dead = (m_new == -INFINITY);
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      // P overwrites the first ABN/2 columns of this buffer as packed bf16
      // pairs.  PV(j-2) read the buffer's previous P before QK(j) wrote S
      // (MMAs of one issuing thread execute in order), so they are free.
#pragma unroll
      for (int c = 0; c < NCK; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float x0 = fmaf(__uint_as_float(u[c][i]), sl2, -m_new);
          const float x1 = fmaf(__uint_as_float(u[c][i + 1]), sl2, -m_new);
          const float p0 = dead ? 0.f : ex2_approx(x0);
          const float p1 = dead ? 0.f : ex2_approx(x1);
          sum4[(i >> 1) & 3] += p0 + p1;
          pk[i >> 1] = pack_bf16(p0, p1);
        }
        tmem_st16(tS + c * 16, pk);
      }
      const float rowsum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
      __syncwarp();
      // O and the P columns are busy until PV(j-1) of this tile completes.
      if (j > 0) {
        if (!mbar_wait(&o_done[t], (j - 1) & 1, err, kErrTimeoutSoftmax)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow && m_ref != -INFINITY)) {
          const float a = (grow && m_ref != -INFINITY) ? exp2f(m_ref - m_new) : 1.f;
#pragma unroll
          for (int c = 0; c < D; c += 32) {
            uint32_t o[32];
            tmem_ld32(tO + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * a);
            tmem_st32(tO + c, o);
          }
        }
      }
      const float alpha = (m_ref == -INFINITY) ? 0.f : (grow ? exp2f(m_ref - m_new) : 1.f);
      l = l * alpha + rowsum;
      m_ref = m_new;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    // --------------------------------------------------------- epilogue
    if (ok && n_kblk > 0 && mbar_wait(&o_done[t], (n_kblk - 1) & 1, err, kErrTimeoutSoftmax)) {
      tc_fence_after();
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      const bool row_ok = qi < S;
      __nv_bfloat16* orow = args.O + (static_cast<int64_t>(tok0 + qi) * args.Hq + h) * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t o[32];
        tmem_ld32(tO + c, o);
        tmem_wait_ld();
        if (row_ok) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(o[q * 8 + 0]) * inv_l, __uint_as_float(o[q * 8 + 1]) * inv_l);
            v.y = pack_bf16(__uint_as_float(o[q * 8 + 2]) * inv_l, __uint_as_float(o[q * 8 + 3]) * inv_l);
            v.z = pack_bf16(__uint_as_float(o[q * 8 + 4]) * inv_l, __uint_as_float(o[q * 8 + 5]) * inv_l);
            v.w = pack_bf16(__uint_as_float(o[q * 8 + 6]) * inv_l, __uint_as_float(o[q * 8 + 7]) * inv_l);
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
// Key/value source for context parallelism: kv [B*Sk, 2*Hk*D] (k | v per row)
// and the query offsets (see AttnArgs).
struct AttnKV {
  const torch::Tensor* kv = nullptr;
  int Sk = 0, off0 = 0, off1 = 0, split = 0;
  const unsigned* kv_flags = nullptr;
  unsigned kv_seq = 0;
  int cp_c = 1, cp_world = 1;
  const int* kv_lo = nullptr;  // key-range mask (self-attention only)
};

template <int D>
static void launch_attn_fwd(const torch::Tensor& qk, const torch::Tensor& qkv, torch::Tensor& o,
                            torch::Tensor& lse, int B, int S, int Hq, int Hk, bool causal, float scale,
                            const AttnKV& cp = AttnKV()) {
  using L = AttnFwdSmem<D>;
  const int64_t T = static_cast<int64_t>(B) * S;
  auto tq = make_tmap_3d_bf16(qk.data_ptr(), D, Hq + Hk, T, D, (int64_t)(Hq + Hk) * D, 64, 1, ABM);
  CUtensorMap tv, tk;
  AttnArgs a;
  if (cp.kv != nullptr) {
    const int64_t Tk = static_cast<int64_t>(B) * cp.Sk;
    tk = make_tmap_3d_bf16(cp.kv->data_ptr(), D, 2 * Hk, Tk, D, (int64_t)(2 * Hk) * D, 64, 1, ABN);
    tv = tk;
    a.Sk = cp.Sk; a.k_head = 0; a.v_head = Hk;
    a.off0 = cp.off0; a.off1 = cp.off1; a.split = cp.split;
    a.kv_flags = cp.kv_flags; a.kv_seq = cp.kv_seq; a.cp_c = cp.cp_c; a.cp_world = cp.cp_world;
  } else {
    a.kv_flags = nullptr; a.kv_seq = 0; a.cp_c = 1; a.cp_world = 1;
    tv = make_tmap_3d_bf16(qkv.data_ptr(), D, Hq + 2 * Hk, T, D, (int64_t)(Hq + 2 * Hk) * D, 64, 1, ABN);
    tk = make_tmap_3d_bf16(qk.data_ptr(), D, Hq + Hk, T, D, (int64_t)(Hq + Hk) * D, 64, 1, ABN);  // ABN-row boxes
    a.Sk = S; a.k_head = Hq; a.v_head = Hq + Hk;
    a.off0 = 0; a.off1 = 0; a.split = S;
  }
  a.kv_lo = cp.kv_lo;
  a.B = B; a.S = S; a.Hq = Hq; a.Hk = Hk;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal = causal ? 1 : 0;
  a.O = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.err = error_flag_ptr();
  auto kern = attn_fwd_kernel<D>;
  set_max_smem_once(reinterpret_cast<const void*>(kern), L::kBytes);
  const int grid = B * Hq * ((S + ABM * kTilesPerCta - 1) / (ABM * kTilesPerCta));
  kern<<<grid, kAttnThreads, L::kBytes, at::cuda::getCurrentCUDAStream()>>>(tq, tv, tk, a);
  NQ_CHECK_CUDA(cudaGetLastError());
}

std::vector<torch::Tensor> attn_fwd(torch::Tensor qk, torch::Tensor qkv, int64_t B, int64_t S,
                                    int64_t Hq, int64_t Hk, int64_t D, bool causal, double scale,
                                    c10::optional<torch::Tensor> kv_lo) {
  check_bf16(qk, "qk"); check_bf16(qkv, "qkv");
  TORCH_CHECK(qk.is_contiguous() && qkv.is_contiguous(), "attn_fwd: contiguous inputs");
  TORCH_CHECK(qk.size(1) == (Hq + Hk) * D && qkv.size(1) == (Hq + 2 * Hk) * D, "attn_fwd: widths");
  TORCH_CHECK(Hq % Hk == 0, "attn_fwd: Hq % Hk");
  c10::cuda::CUDAGuard g(qk.device());
  auto o = torch::empty({B * S, Hq * D}, qk.options());
  auto lse = torch::empty({B, Hq, S}, qk.options().dtype(torch::kFloat32));
  if (B * S == 0) return {o, lse};
  AttnKV self;
  if (kv_lo.has_value() && kv_lo->defined()) {
    TORCH_CHECK(causal, "attn_fwd: the key-range mask applies to causal attention");
    TORCH_CHECK(kv_lo->is_cuda() && kv_lo->scalar_type() == torch::kInt32 && kv_lo->is_contiguous() &&
                    kv_lo->numel() == B * S, "attn_fwd: kv_lo int32 [B*S]");
    self.kv_lo = kv_lo->data_ptr<int>();
  }
  if (D == 128) launch_attn_fwd<128>(qk, qkv, o, lse, B, S, Hq, Hk, causal, (float)scale, self);
  else if (D == 64) launch_attn_fwd<64>(qk, qkv, o, lse, B, S, Hq, Hk, causal, (float)scale, self);
  else TORCH_CHECK(false, "attn_fwd: head_dim must be 64 or 128");
  return {o, lse};
}

// Context-parallel forward: queries of this rank (qk [B*S, (Hq+Hk)*D], two
// chunks of rows [0, split) and [split, S) at key positions +off0 / +off1)
// against gathered keys/values kv [B*Sk, 2*Hk*D]; causal by position.
std::vector<torch::Tensor> attn_fwd_cp(torch::Tensor qk, torch::Tensor kv, int64_t B, int64_t S, int64_t Sk,
                                       int64_t Hq, int64_t Hk, int64_t D, int64_t off0, int64_t off1,
                                       int64_t split, double scale, int64_t kv_flags, int64_t kv_seq,
                                       int64_t cp_world) {
  check_bf16(qk, "qk"); check_bf16(kv, "kv");
  TORCH_CHECK(qk.is_contiguous() && kv.is_contiguous(), "attn_fwd_cp: contiguous inputs");
  TORCH_CHECK(qk.size(1) == (Hq + Hk) * D && kv.size(1) == 2 * Hk * D && kv.size(0) == B * Sk,
              "attn_fwd_cp: shapes");
  TORCH_CHECK(split % (ABM * kTilesPerCta) == 0 && S % (ABM * kTilesPerCta) == 0,
              "attn_fwd_cp: chunk lengths must be multiples of 256");
  TORCH_CHECK(off0 >= 0 && off1 >= 0 && off0 + split <= Sk && off1 + S - split <= Sk, "attn_fwd_cp: offsets");
  c10::cuda::CUDAGuard g(qk.device());
  auto o = torch::empty({B * S, Hq * D}, qk.options());
  auto lse = torch::empty({B, Hq, S}, qk.options().dtype(torch::kFloat32));
  if (B * S == 0) return {o, lse};
  AttnKV cp;
  cp.kv = &kv; cp.Sk = static_cast<int>(Sk); cp.off0 = static_cast<int>(off0);
  cp.off1 = static_cast<int>(off1 - split);  // row i >= split sits at off1 + (i - split)
  cp.split = static_cast<int>(split);
  if (kv_flags != 0) {
    TORCH_CHECK(cp_world >= 1 && cp_world <= 8 && Sk % (2 * cp_world) == 0 && (Sk / (2 * cp_world)) % ABN == 0,
                "attn_fwd_cp: zigzag chunks must be multiples of the key block");
    cp.kv_flags = reinterpret_cast<const unsigned*>(kv_flags);
    cp.kv_seq = static_cast<unsigned>(kv_seq);
    cp.cp_world = static_cast<int>(cp_world);
    cp.cp_c = static_cast<int>(Sk / (2 * cp_world));
  }
  if (D == 128) launch_attn_fwd<128>(qk, qk, o, lse, B, S, Hq, Hk, true, (float)scale, cp);
  else if (D == 64) launch_attn_fwd<64>(qk, qk, o, lse, B, S, Hq, Hk, true, (float)scale, cp);
  else TORCH_CHECK(false, "attn_fwd_cp: head_dim must be 64 or 128");
  return {o, lse};
}

}  // namespace nq
