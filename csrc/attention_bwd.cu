// Flash-attention backward for sm_100a (tcgen05 + TMEM + TMA).
//
// CTA = (batch, kv-head, 128-key block), 12 warps.  K and V stay resident in
// shared memory; the CTA walks every q-head of its GQA group and every query
// block that can see its keys (causal).  Per (q-head, query block) it issues
//   S^T  = K Q^T        -> TMEM cols [0,128)     (thread = key row)
//   dP^T = V dO^T       -> TMEM cols [128,256)
//   compute: P^T = exp2(S^T*scale*log2e - lse*log2e) written back into TMEM as
//            packed bf16 over S^T; dS^T = P^T (dP^T - delta) * scale written to a
//            128B-swizzled shared tile
//   dV  += P^T dO       (A operand P^T read from TMEM)   TMEM [384,512)
//   dK  += dS^T Q                                        TMEM [256,384)
//   dQ_i = dS K         -> TMEM cols [128,256) (over dP^T, already consumed);
//          the dS^T tile written K-major for dK is read MN-major as dQ's A
//          operand (same swizzled bytes), so there is no transpose pass.
// Warp 0 streams Q/dO through a 2-deep ring, warp 1 issues the MMAs, warps 4-7
// and 8-11 are two compute warpgroups that split every tile's 128 columns
// (q columns for P/dS, head-dim columns for dQ/dK/dV).  dQ_i is staged (fp32,
// 128B-swizzled) in iteration i's Q/dO buffers once its MMAs are done, and warp 2
// adds it into an fp32 buffer with TMA bulk reductions
// (cp.reduce.async.bulk.tensor .add) off the compute warps' critical path; the
// producer reuses the buffers after that reduction has read them.  Warp 3
// prefetches the next iteration's lse / delta.  The fp32 dq buffer is zeroed by
// the pre-pass kernel, which also computes delta = rowsum(dO * O).
// Outputs: dq|dk fp32 [T, (Hq+Hk)*D]; dv bf16 written into the v slot of dqkv.
//
// That serial schedule is kept for head_dim 64.  head_dim 128 runs
// attn_bwd_pp_kernel (below): 64-query iterations alternate between the two
// warpgroups, each with its own S^T / dP^T region in TMEM, so the tensor pipe
// works on one warpgroup's iteration while the other computes P^T / dS^T
// (4 x 4096 tokens, 16/8 heads: 1159 -> 1067 us on B200; 984 us with the
// grouped heaviest-first block order; 926 us with dQ^T issued ahead of dV/dK).
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace nq {

constexpr int BKN = 128;  // keys per CTA
constexpr int BQM = 128;  // queries per iteration
constexpr int kBwdThreads = 384;

template <int D>
struct AttnBwdSmem {
  static constexpr int kTile = 128 * D * 2;  // K, V, Q, dO tiles
  static constexpr int kDS = BKN * BQM * 2;
  static constexpr int kKOff = 0;
  static constexpr int kVOff = kKOff + kTile;
  static constexpr int kQOff = kVOff + kTile;        // [2]
  static constexpr int kDOOff = kQOff + 2 * kTile;    // [2]
  static constexpr int kDSOff = kDOOff + 2 * kTile;
  static constexpr int kLseOff = kDSOff + kDS;        // 128 lse (log2 units) + 128 delta
  static constexpr int kBarOff = kLseOff + 2 * BQM * 4;
  static constexpr int kBytes = kBarOff + 128 + 1024;
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
  // Context parallelism (see AttnArgs in attention.cu): keys/values come from
  // a gathered [B*Sk, 2*Hk*D] buffer (heads k_head / v_head of the tmK map);
  // query row i sits at key position i + off0 (i < split) or i + off1; dK and
  // dV of the gathered keys are written in fp32 to dkv_cp [B*Sk, 2*Hk*D].
  // Self-attention: Sk = S, offsets 0, dkv_cp null.
  int Sk, k_head, v_head, off0, off1, split;
  float* dkv_cp;
  // Key-range mask (the forward's kv_lo, seen from the keys): key token j is
  // seen by queries [j, q_hi[j]) of its row; q_hi is non-decreasing along a
  // row, so a key block's last key bounds the query blocks to visit.
  // null: causal only.
  const int* q_hi;
};

__device__ __forceinline__ float bwd_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

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

__device__ __forceinline__ void wg_sync(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }

template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQK, const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmDO, const __grid_constant__ CUtensorMap tmDQ,
                    const __grid_constant__ CUtensorMap tmK, const AttnBwdArgs args) {
  using L = AttnBwdSmem<D>;
  constexpr int KCH = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sDO = smem + L::kDOOff;
  uint8_t* sDS = smem + L::kDSOff;
  float* sLse = reinterpret_cast<float*>(smem + L::kLseOff);
  float* sDelta = sLse + BQM;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;     // S^T and dP^T ready
  uint64_t* pt_full = bars + 6;    // P^T (TMEM) / dS^T (SMEM) written; S^T, dP^T consumed (8 warps)
  uint64_t* dq_full = bars + 7;    // dQ_i in TMEM; dS^T smem free again
  uint64_t* dq_free = bars + 8;    // dQ_i drained (8 warps)
  uint64_t* acc_done = bars + 9;   // final dK / dV
  uint64_t* staged = bars + 10;    // dQ_i staged in the Q/dO buffer of iteration i (8 warps)
  uint64_t* qdo_rel = bars + 11;   // [2] bulk reduce finished reading the staged dQ
  uint64_t* lse_rdy = bars + 13;   // lse/delta of the next iteration in shared memory
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = args.err;
  const int S = args.S;
  const int Sk = args.Sk;
  const int n_kblk = (Sk + BKN - 1) / BKN;
  // Head-major order: the key blocks of one (batch, kv-head) run side by side
  // and share its streamed Q / dO / LSE tiles in L2 (measured faster than a
  // heaviness-major order here); within a head the heaviest (lowest) key
  // blocks start first.
  const int nb = static_cast<int>(blockIdx.x) % n_kblk;
  const int bk = static_cast<int>(blockIdx.x) / n_kblk;
  const int b = bk / args.Hk;
  const int hk = bk - b * args.Hk;
  const int G = args.Hq / args.Hk;
  const int k0 = nb * BKN;
  const int tok0 = b * S;
  const int ktok0 = b * Sk;
  const int n_mblk = (S + BQM - 1) / BQM;
  // Query blocks that can see this key block, per query chunk: chunk 0 covers
  // blocks [0, split/BQM) at offset off0, chunk 1 the rest at offset off1.
  const int split_mb = (args.split + BQM - 1) / BQM;
  int b0 = 0, e0 = split_mb, b1 = split_mb, e1 = n_mblk;
  if (args.q_hi != nullptr) e0 = min(e0, (args.q_hi[ktok0 + min(k0 + BKN, Sk) - 1] + BQM - 1) / BQM);
  if (args.causal) {
    // first block with a query at key position >= k0 (floor division of possibly negative values)
    const int f0 = k0 - args.off0, f1 = k0 - args.off1;
    b0 = max(b0, f0 >= 0 ? f0 / BQM : 0);
    b1 = max(b1, f1 >= 0 ? f1 / BQM : 0);
  }
  const int n0 = max(0, e0 - b0), n1 = max(0, e1 - b1);
  const int iters_per_head = n0 + n1;
  const int n_iter = G * iters_per_head;

  if (warp == 0 && lane == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qdo_full[s], 1);
      mbar_init(&qdo_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(pt_full, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 8);
    mbar_init(acc_done, 1);
    mbar_init(staged, 8);
    mbar_init(&qdo_rel[0], 1);
    mbar_init(&qdo_rel[1], 1);
    mbar_init(lse_rdy, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmDQ);
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
  const uint32_t tST = tmem;         // S^T, then P^T (bf16 packed in cols [0,64))
  const uint32_t tDP = tmem + 128;   // dP^T, then dQ
  const uint32_t tDK = tmem + 256;
  const uint32_t tDV = tmem + 384;

  auto iter_coords = [&](int it, int& hq, int& mb) {
    const int g = it / iters_per_head;
    hq = hk * G + g;
    const int l = it - g * iters_per_head;
    mb = (l < n0) ? b0 + l : b1 + (l - n0);
  };
  auto qoff_of = [&](int q0) { return (q0 < args.split) ? args.off0 : args.off1; };

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * L::kTile);
#pragma unroll
      for (int c = 0; c < KCH; ++c) {
        tma_load_3d(sK + c * 128 * 128, &tmK, kv_full, c * 64, args.k_head + hk, ktok0 + k0);
        tma_load_3d(sV + c * 128 * 128, &tmV, kv_full, c * 64, args.v_head + hk, ktok0 + k0);
      }
      for (int it = 0; it < n_iter; ++it) {
        int hq, mb;
        iter_coords(it, hq, mb);
        const int bf = it & 1;
        // buffer bf is reused once iteration it-2's MMAs and its dQ reduction are done
        if (!mbar_wait(&qdo_empty[bf], ((it >> 1) & 1) ^ 1, err, kErrTimeoutProducer)) break;
        if (!mbar_wait(&qdo_rel[bf], ((it >> 1) & 1) ^ 1, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&qdo_full[bf], 2 * L::kTile);
#pragma unroll
        for (int c = 0; c < KCH; ++c) {
          tma_load_3d(sQ + bf * L::kTile + c * 128 * 128, &tmQK, &qdo_full[bf], c * 64, hq, tok0 + mb * BQM);
          tma_load_3d(sDO + bf * L::kTile + c * 128 * 128, &tmDO, &qdo_full[bf], c * 64, hq, tok0 + mb * BQM);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t id_s = idesc_bf16(BKN, BQM, false, false);   // K Q^T, V dO^T
      constexpr uint32_t id_kv = idesc_bf16(BKN, D, false, true);     // P^T dO, dS^T Q
      constexpr uint32_t id_q = idesc_bf16(BQM, D, true, true);       // dS K
      bool ok = mbar_wait(kv_full, 0, err, kErrTimeoutMma);
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aDS = smem_u32(sDS);
      for (int it = 0; it < n_iter && ok; ++it) {
        const int bf = it & 1;
        const uint32_t aQ = smem_u32(sQ + bf * L::kTile), aDO = smem_u32(sDO + bf * L::kTile);
        if (!mbar_wait(&qdo_full[bf], (it >> 1) & 1, err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        // S^T (tST is free: P^T(it-1) was read by dV(it-1), issued earlier on this thread)
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          umma_bf16(tST, sdesc_sw128(aK + off, 16, 1024), sdesc_sw128(aQ + off, 16, 1024), id_s, kk > 0);
        }
        // dP^T overwrites dQ(it-1): wait until the compute warps drained it
        if (!mbar_wait(dq_free, (it & 1) ^ 1, err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          umma_bf16(tDP, sdesc_sw128(aV + off, 16, 1024), sdesc_sw128(aDO + off, 16, 1024), id_s, kk > 0);
        }
        umma_commit(s_full);
        if (!mbar_wait(pt_full, it & 1, err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQM / 16; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          // dV += P^T dO : A = P^T from TMEM (K = queries), B = dO MN-major
          umma_bf16_ts(tDV, tST + kk * 8, sdesc_sw128(aDO + kk * 2048, 128 * 128, 1024), id_kv, acc);
          // dK += dS^T Q : A = dS^T smem K-major, B = Q MN-major
          umma_bf16(tDK, sdesc_sw128(aDS + (kk >> 2) * (128 * 128) + (kk & 3) * 32, 16, 1024),
                    sdesc_sw128(aQ + kk * 2048, 128 * 128, 1024), id_kv, acc);
        }
        // dQ = dS K (M = queries, K = keys): A = dS^T tile read MN-major, B = K MN-major
#pragma unroll
        for (int kk = 0; kk < BKN / 16; ++kk) {
          umma_bf16(tDP, sdesc_sw128(aDS + kk * 2048, 128 * 128, 1024),
                    sdesc_sw128(aK + kk * 2048, 128 * 128, 1024), id_q, kk > 0);
        }
        umma_commit(dq_full);
        umma_commit(&qdo_empty[bf]);
      }
      if (ok) umma_commit(acc_done);
    }
  } else if (warp == 2) {
    // ------------------------------------------------ dQ bulk-reduce issuer
    if (elect_one()) {
      for (int it = 0; it < n_iter; ++it) {
        int hq, mb;
        iter_coords(it, hq, mb);
        const int bf = it & 1;
        if (!mbar_wait(staged, it & 1, err, kErrTimeoutDrain)) break;
#pragma unroll
        for (int bx = 0; bx < D / 32; ++bx) {
          const uint8_t* src = (D == 128) ? ((bx < 2 ? sQ : sDO) + bf * L::kTile + (bx & 1) * (128 * 128))
                                          : ((bx == 0 ? sQ : sDO) + bf * L::kTile);
          tma_reduce_add_3d(&tmDQ, src, 32 * bx, hq, tok0 + mb * BQM);
        }
        bulk_commit();
        bulk_wait_read_all();
        mbar_arrive(&qdo_rel[bf]);
      }
      bulk_wait_all();
    }
  } else if (warp == 3) {
    // ------------------------------------- lse / delta prefetch (per iteration)
    for (int it = 0; it < n_iter; ++it) {
      int hq, mb;
      iter_coords(it, hq, mb);
      // the previous iteration's P/dS phase is the only reader of these values
      if (it > 0 && !mbar_wait(pt_full, (it - 1) & 1, err, kErrTimeoutDrain)) break;
      const int q0 = mb * BQM;
#pragma unroll
      for (int e = 0; e < BQM / 32; ++e) {
        const int ql = e * 32 + lane;
        const int q = q0 + ql;
        const int64_t idx = (static_cast<int64_t>(b) * args.Hq + hq) * S + q;
        sLse[ql] = (q < S) ? args.lse[idx] * 1.4426950408889634f : INFINITY;
        sDelta[ql] = (q < S) ? args.delta[idx] : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(lse_rdy);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------- compute WGs
    const int wg = (warp - 4) >> 2;     // column half
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane: key row (P/dS phase) or query row (dQ phase)
    const int col0 = wg * 64;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int kj = k0 + r;              // this thread's key position
    const int qhi = (args.q_hi != nullptr) ? args.q_hi[ktok0 + min(kj, Sk - 1)] : 0x7fffffff;
    bool ok = true;
    for (int it = 0; it < n_iter; ++it) {
      int hq, mb;
      iter_coords(it, hq, mb);
      const uint32_t ph = it & 1;
      const int q0 = mb * BQM;
      if (!mbar_wait(lse_rdy, ph, err, kErrTimeoutSoftmax)) { ok = false; break; }
      if (!mbar_wait(s_full, ph, err, kErrTimeoutSoftmax)) { ok = false; break; }
      tc_fence_after();
      const int qoff = qoff_of(q0);
      const bool need_mask = (args.causal && k0 + BKN - 1 > q0 + qoff) || (q0 + BQM > S) || (k0 + BKN > Sk) ||
                             (q0 + BQM > qhi);
      uint32_t us2[2][32], ud2[2][32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld32(tST + lane_base + col0 + 32 * c, us2[c]);
        tmem_ld32(tDP + lane_base + col0 + 32 * c, ud2[c]);
      }
      tmem_wait_ld();
      // P^T of the second column half lands in TMEM columns the first half is
      // still reading as S^T: both compute warpgroups finish loading first.
      asm volatile("bar.sync 3, 256;" ::: "memory");
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        const uint32_t* us = us2[c >> 5];
        const uint32_t* ud = ud2[c >> 5];
        float p[32], ds[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(sLse + col0 + c + i);
          const float4 d4 = *reinterpret_cast<const float4*>(sDelta + col0 + c + i);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
          const float dl[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float pv = bwd_ex2(fmaf(__uint_as_float(us[i + e]), args.scale_log2, -lv[e]));
            p[i + e] = pv;
            ds[i + e] = pv * (__uint_as_float(ud[i + e]) - dl[e]) * args.scale;
          }
        }
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int qi = q0 + col0 + c + i;
            const bool m = (qi >= S) || (kj >= Sk) || (args.causal && kj > qi + qoff) || (qi >= qhi);
            p[i] = m ? 0.f : p[i];
            ds[i] = m ? 0.f : ds[i];
          }
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(p[2 * i], p[2 * i + 1]);
        // P^T as packed bf16 over the first 64 columns of the S^T region:
        // query column q lands in TMEM column q / 2.
        tmem_st16(tST + lane_base + (col0 + c) / 2, pk);
#pragma unroll
        for (int i = 0; i < 32; i += 8) store8_sw128(sDS, r, col0 + c + i, &ds[i]);
      }
      tmem_wait_st();
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pt_full);
      // dQ drain: TMEM -> fp32 staging in the dS tile (free once the dQ MMA
      // completed, which dq_full implies) -> TMA bulk reduce-add into the fp32 dq
      // buffer.  Rounds of 64 head-dim columns; each warpgroup stages one
      // 128-row x 32-column box (128B-swizzled, bank-conflict free).
      if (!mbar_wait(dq_full, ph, err, kErrTimeoutSoftmax)) { ok = false; break; }
      tc_fence_after();
      {
        const int bf = it & 1;
        uint32_t u[D / 64][32];
#pragma unroll
        for (int hh = 0; hh < D / 64; ++hh) tmem_ld32(tDP + lane_base + 64 * hh + 32 * wg, u[hh]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_free);  // TMEM region free for the next dP^T
        // dQ box (hh, wg) = 128 rows x 32 fp32 columns, 128B-swizzled, into the
        // Q/dO buffer of this iteration (all of this iteration's MMAs are done).
#pragma unroll
        for (int hh = 0; hh < D / 64; ++hh) {
          const int bx = 2 * hh + wg;
          uint8_t* box = (D == 128) ? ((bx < 2 ? sQ : sDO) + bf * L::kTile + (bx & 1) * (128 * 128))
                                    : ((bx == 0 ? sQ : sDO) + bf * L::kTile);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4*>(box + r * 128 + ((q ^ (r & 7)) << 4)) =
                make_uint4(u[hh][4 * q], u[hh][4 * q + 1], u[hh][4 * q + 2], u[hh][4 * q + 3]);
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(staged);
      }
    }
    // ------------------------------------------------------- dK / dV out
    if (ok && n_iter > 0 && mbar_wait(acc_done, 0, err, kErrTimeoutSoftmax)) {
      tc_fence_after();
      const bool row_ok = kj < Sk;
      const bool cp = args.dkv_cp != nullptr;
      float* dk = cp ? args.dkv_cp + (static_cast<int64_t>(ktok0 + kj) * (2 * args.Hk) + hk) * D
                     : args.dqk + (static_cast<int64_t>(tok0 + kj) * (args.Hq + args.Hk) + args.Hq + hk) * D;
      float* dv_cp = cp ? args.dkv_cp + (static_cast<int64_t>(ktok0 + kj) * (2 * args.Hk) + args.Hk + hk) * D
                        : nullptr;
      __nv_bfloat16* dv = cp ? nullptr
                             : args.dqkv + (static_cast<int64_t>(tok0 + kj) * (args.Hq + 2 * args.Hk) + args.Hq + args.Hk + hk) * D;
#pragma unroll
      for (int c = 0; c < D / 2; c += 32) {
        const int cc = (D / 2) * wg + c;
        uint32_t uk[32], uv[32];
        tmem_ld32(tDK + lane_base + cc, uk);
        tmem_ld32(tDV + lane_base + cc, uv);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dk + cc + i) = make_float4(__uint_as_float(uk[i]), __uint_as_float(uk[i + 1]),
                                                                __uint_as_float(uk[i + 2]), __uint_as_float(uk[i + 3]));
          if (cp) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dv_cp + cc + i) = make_float4(__uint_as_float(uv[i]), __uint_as_float(uv[i + 1]),
                                                                       __uint_as_float(uv[i + 2]), __uint_as_float(uv[i + 3]));
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 v;
              v.x = pack_bf16(__uint_as_float(uv[q * 8 + 0]), __uint_as_float(uv[q * 8 + 1]));
              v.y = pack_bf16(__uint_as_float(uv[q * 8 + 2]), __uint_as_float(uv[q * 8 + 3]));
              v.z = pack_bf16(__uint_as_float(uv[q * 8 + 4]), __uint_as_float(uv[q * 8 + 5]));
              v.w = pack_bf16(__uint_as_float(uv[q * 8 + 6]), __uint_as_float(uv[q * 8 + 7]));
              reinterpret_cast<uint4*>(dv + cc)[q] = v;
            }
          }
        }
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

// ---------------------------------------------------------------------------
// head_dim 128: ping-pong schedule over 64-query iterations.
//
// The serial schedule above leaves the tensor pipe idle while the compute
// warpgroups turn S^T / dP^T into P^T / dS^T (about 60% of an iteration on
// B200).  Here warpgroup w owns iterations it with it % 2 == w and its own
// TMEM region: S^T[w] (128 keys x 64 queries) and dP^T[w] (then dQ^T[w] =
// K^T dS^T, 128 head dims x 64 queries) in columns [128w, 128w + 128); dK and
// dV keep columns [256, 512).  The MMA warp issues S^T/dP^T of iteration it+1
// before it waits for iteration it's P^T/dS^T, so one warpgroup's exp / dS
// work runs while the tensor pipe serves the other.  Q/dO stream through a
// 4-deep ring of 64-row tiles; dQ^T is staged (fp32, 128B-swizzled, query
// rows) in the iteration's Q/dO stage and added into the fp32 dq buffer with
// TMA bulk reductions by warp 2.  Warp 3 prefetches lse / delta per warpgroup.
constexpr int PBQ = 64;    // queries per iteration
constexpr int PNS = 4;     // Q/dO ring depth

struct AttnBwdPPSmem {
  static constexpr int kKV = 128 * 128 * 2;    // K or V tile: 2 regions of 128 rows x 128 B
  static constexpr int kQT = PBQ * 128 * 2;    // Q or dO tile: 2 regions of 64 rows x 128 B
  static constexpr int kDS = 128 * PBQ * 2;    // dS^T tile: 128 key rows x 128 B
  static constexpr int kKOff = 0;
  static constexpr int kVOff = kKOff + kKV;
  static constexpr int kStageOff = kVOff + kKV;             // [PNS] x (Q | dO)
  static constexpr int kDSOff = kStageOff + PNS * 2 * kQT;  // [2]
  static constexpr int kLseOff = kDSOff + 2 * kDS;          // [2] x (64 lse + 64 delta)
  static constexpr int kBarOff = kLseOff + 2 * 2 * PBQ * 4;
  static constexpr int kBytes = kBarOff + 256 + 1024;
};

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_pp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmDO, const __grid_constant__ CUtensorMap tmDQ,
                       const __grid_constant__ CUtensorMap tmK, const AttnBwdArgs args) {
  using L = AttnBwdPPSmem;
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  auto sQ = [&](int s) { return smem + L::kStageOff + s * 2 * L::kQT; };
  auto sDO = [&](int s) { return smem + L::kStageOff + s * 2 * L::kQT + L::kQT; };
  auto sDS = [&](int w) { return smem + L::kDSOff + w * L::kDS; };
  auto sLse = [&](int w) { return reinterpret_cast<float*>(smem + L::kLseOff) + w * 2 * PBQ; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;    // [PNS]
  uint64_t* qdo_empty = bars + 5;   // [PNS] this iteration's MMAs are done with Q/dO
  uint64_t* qdo_rel = bars + 9;     // [PNS] the bulk reduce has read the staged dQ
  uint64_t* staged = bars + 13;     // [PNS] dQ staged in the stage (4 warps)
  uint64_t* s_full = bars + 17;     // [2] S^T[w], dP^T[w] in TMEM
  uint64_t* pds_ready = bars + 19;  // [2] P^T[w] in TMEM, dS^T[w] in SMEM (4 warps)
  uint64_t* dq_full = bars + 21;    // [2] dQ^T[w] in TMEM
  uint64_t* dq_free = bars + 23;    // [2] dQ^T[w] drained (4 warps)
  uint64_t* lse_rdy = bars + 25;    // [2]
  uint64_t* acc_done = bars + 27;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 28);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = args.err;
  const int S = args.S;
  const int Sk = args.Sk;
  const int n_kblk = (Sk + BKN - 1) / BKN;
  // Block order: (batch, kv-head) pairs in groups of 8; inside a group the
  // heaviest (lowest) key blocks of all 8 pairs start first.  The 8 pairs'
  // Q/dO/lse stay L2-resident while the group runs, and the light blocks of
  // the last group fill the tail.
  int nb, bk;
  {
    const int n_pairs = args.B * args.Hk;
    const int grp = static_cast<int>(blockIdx.x) / (8 * n_kblk);
    const int sz = min(8, n_pairs - 8 * grp);
    const int r = static_cast<int>(blockIdx.x) - grp * 8 * n_kblk;
    nb = r / sz;
    bk = 8 * grp + r % sz;
  }
  const int b = bk / args.Hk;
  const int hk = bk - b * args.Hk;
  const int G = args.Hq / args.Hk;
  const int k0 = nb * BKN;
  const int tok0 = b * S;
  const int ktok0 = b * Sk;
  const int n_mblk = (S + PBQ - 1) / PBQ;
  const int split_mb = (args.split + PBQ - 1) / PBQ;
  int b0 = 0, e0 = split_mb, b1 = split_mb, e1 = n_mblk;
  if (args.q_hi != nullptr) e0 = min(e0, (args.q_hi[ktok0 + min(k0 + BKN, Sk) - 1] + PBQ - 1) / PBQ);
  if (args.causal) {
    const int f0 = k0 - args.off0, f1 = k0 - args.off1;
    b0 = max(b0, f0 >= 0 ? f0 / PBQ : 0);
    b1 = max(b1, f1 >= 0 ? f1 / PBQ : 0);
  }
  const int n0 = max(0, e0 - b0), n1 = max(0, e1 - b1);
  const int iters_per_head = n0 + n1;
  const int n_iter = G * iters_per_head;

  if (warp == 0 && lane == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < PNS; ++s) {
      mbar_init(&qdo_full[s], 1);
      mbar_init(&qdo_empty[s], 1);
      mbar_init(&qdo_rel[s], 1);
      mbar_init(&staged[s], 4);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&s_full[w], 1);
      mbar_init(&pds_ready[w], 4);
      mbar_init(&dq_full[w], 1);
      mbar_init(&dq_free[w], 4);
      mbar_init(&lse_rdy[w], 1);
    }
    mbar_init(acc_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmDQ);
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
  const uint32_t tDK = tmem + 256;
  const uint32_t tDV = tmem + 384;

  auto iter_coords = [&](int it, int& hq, int& mb) {
    const int g = it / iters_per_head;
    hq = hk * G + g;
    const int l = it - g * iters_per_head;
    mb = (l < n0) ? b0 + l : b1 + (l - n0);
  };
  auto qoff_of = [&](int q0) { return (q0 < args.split) ? args.off0 : args.off1; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * L::kKV);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tma_load_3d(sK + c * 128 * 128, &tmK, kv_full, c * 64, args.k_head + hk, ktok0 + k0);
        tma_load_3d(sV + c * 128 * 128, &tmV, kv_full, c * 64, args.v_head + hk, ktok0 + k0);
      }
      for (int it = 0; it < n_iter; ++it) {
        int hq, mb;
        iter_coords(it, hq, mb);
        const int s = it % PNS;
        const uint32_t u = static_cast<uint32_t>(it / PNS) & 1;
        if (!mbar_wait(&qdo_empty[s], u ^ 1, err, kErrTimeoutProducer)) break;
        if (!mbar_wait(&qdo_rel[s], u ^ 1, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&qdo_full[s], 2 * L::kQT);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(sQ(s) + c * PBQ * 128, &tmQ, &qdo_full[s], c * 64, hq, tok0 + mb * PBQ);
          tma_load_3d(sDO(s) + c * PBQ * 128, &tmDO, &qdo_full[s], c * 64, hq, tok0 + mb * PBQ);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t id_s = idesc_bf16(BKN, PBQ, false, false);  // K Q^T, V dO^T (keys x queries)
      constexpr uint32_t id_kv = idesc_bf16(BKN, D, false, true);    // P^T dO, dS^T Q (keys x head dims)
      constexpr uint32_t id_q = idesc_bf16(D, PBQ, true, true);      // K^T dS^T (head dims x queries)
      bool ok = mbar_wait(kv_full, 0, err, kErrTimeoutMma);
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV);
      // S^T[w] = K Q^T and dP^T[w] = V dO^T of iteration j (w = j % 2)
      auto issue_sdp = [&](int j) -> bool {
        const int w = j & 1, s = j % PNS;
        if (!mbar_wait(&qdo_full[s], static_cast<uint32_t>(j / PNS) & 1, err, kErrTimeoutMma)) return false;
        // dP^T[w] is where dQ^T of iteration j-2 waits to be drained
        if (!mbar_wait(&dq_free[w], static_cast<uint32_t>((j >> 1) & 1) ^ 1, err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t aQ = smem_u32(sQ(s)), aDO = smem_u32(sDO(s));
        const uint32_t tS = tmem + 128 * w, tP = tS + 64;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t oa = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          const uint32_t ob = (kk >> 2) * (PBQ * 128) + (kk & 3) * 32;
          umma_bf16(tS, sdesc_sw128(aK + oa, 16, 1024), sdesc_sw128(aQ + ob, 16, 1024), id_s, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t oa = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          const uint32_t ob = (kk >> 2) * (PBQ * 128) + (kk & 3) * 32;
          umma_bf16(tP, sdesc_sw128(aV + oa, 16, 1024), sdesc_sw128(aDO + ob, 16, 1024), id_s, kk > 0);
        }
        umma_commit(&s_full[w]);
        return true;
      };
      if (ok && n_iter > 0) ok = issue_sdp(0);
      for (int it = 0; it < n_iter && ok; ++it) {
        const int w = it & 1, s = it % PNS;
        if (it + 1 < n_iter && !issue_sdp(it + 1)) { ok = false; break; }
        if (!mbar_wait(&pds_ready[w], static_cast<uint32_t>(it >> 1) & 1, err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aQ = smem_u32(sQ(s)), aDO = smem_u32(sDO(s)), aDS = smem_u32(sDS(w));
        const uint32_t tS = tmem + 128 * w, tP = tS + 64;
        // dQ^T = K^T dS^T (M = head dims, N = queries, K = keys): A = K read
        // MN-major, B = dS^T read MN-major; lands over the consumed dP^T[w].
        // Issued first so the warpgroup can drain it while dV / dK run.
#pragma unroll
        for (int kk = 0; kk < BKN / 16; ++kk) {
          umma_bf16(tP, sdesc_sw128(aK + kk * 2048, 128 * 128, 1024), sdesc_sw128(aDS + kk * 2048, L::kDS, 1024),
                    id_q, kk > 0);
        }
        umma_commit(&dq_full[w]);
#pragma unroll
        for (int kk = 0; kk < PBQ / 16; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          // dV += P^T dO : A = P^T from TMEM (K = queries), B = dO MN-major
          umma_bf16_ts(tDV, tS + kk * 8, sdesc_sw128(aDO + kk * 2048, PBQ * 128, 1024), id_kv, acc);
          // dK += dS^T Q : A = dS^T smem K-major, B = Q MN-major
          umma_bf16(tDK, sdesc_sw128(aDS + kk * 32, 16, 1024), sdesc_sw128(aQ + kk * 2048, PBQ * 128, 1024),
                    id_kv, acc);
        }
        umma_commit(&qdo_empty[s]);
      }
      if (ok) umma_commit(acc_done);
    }
  } else if (warp == 2) {
    // ------------------------------------------------ dQ bulk-reduce issuer
    if (elect_one()) {
      for (int it = 0; it < n_iter; ++it) {
        int hq, mb;
        iter_coords(it, hq, mb);
        const int s = it % PNS;
        if (!mbar_wait(&staged[s], static_cast<uint32_t>(it / PNS) & 1, err, kErrTimeoutDrain)) break;
#pragma unroll
        for (int bx = 0; bx < D / 32; ++bx)
          tma_reduce_add_3d(&tmDQ, (bx < 2 ? sQ(s) : sDO(s)) + (bx & 1) * (PBQ * 128), 32 * bx, hq, tok0 + mb * PBQ);
        bulk_commit();
        bulk_wait_read_all();
        mbar_arrive(&qdo_rel[s]);
      }
      bulk_wait_all();
    }
  } else if (warp == 3) {
    // ------------------------------------- lse / delta prefetch (per iteration)
    for (int it = 0; it < n_iter; ++it) {
      int hq, mb;
      iter_coords(it, hq, mb);
      const int w = it & 1;
      // warpgroup w read these values for iteration it-2 before publishing P/dS
      if (it >= 2 && !mbar_wait(&pds_ready[w], static_cast<uint32_t>((it - 2) >> 1) & 1, err, kErrTimeoutDrain)) break;
      const int q0 = mb * PBQ;
      float* lse = sLse(w);
#pragma unroll
      for (int e = 0; e < PBQ / 32; ++e) {
        const int ql = e * 32 + lane;
        const int q = q0 + ql;
        const int64_t idx = (static_cast<int64_t>(b) * args.Hq + hq) * S + q;
        lse[ql] = (q < S) ? args.lse[idx] * 1.4426950408889634f : INFINITY;
        lse[PBQ + ql] = (q < S) ? args.delta[idx] : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&lse_rdy[w]);
    }
  } else {
    // ------------------------------------------------------- compute WGs
    const int w = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane: key row (P/dS) or head dim (dQ^T)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + 128 * w + lane_base, tP = tS + 64;
    const int kj = k0 + r;
    const int qhi = (args.q_hi != nullptr) ? args.q_hi[ktok0 + min(kj, Sk - 1)] : 0x7fffffff;
    const float* lse = sLse(w);
    const float* dlt = lse + PBQ;
    uint8_t* ds_tile = sDS(w);
    bool ok = true;
    for (int it = w; it < n_iter; it += 2) {
      int hq, mb;
      iter_coords(it, hq, mb);
      const uint32_t ph = static_cast<uint32_t>(it >> 1) & 1;
      const int s = it % PNS;
      const int q0 = mb * PBQ;
      if (!mbar_wait(&lse_rdy[w], ph, err, kErrTimeoutSoftmax)) { ok = false; break; }
      if (!mbar_wait(&s_full[w], ph, err, kErrTimeoutSoftmax)) { ok = false; break; }
      tc_fence_after();
      const int qoff = qoff_of(q0);
      const bool need_mask = (args.causal && k0 + BKN - 1 > q0 + qoff) || (q0 + PBQ > S) || (k0 + BKN > Sk) ||
                             (q0 + PBQ > qhi);
      uint32_t us2[2][32], ud2[2][32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld32(tS + 32 * c, us2[c]);
        tmem_ld32(tP + 32 * c, ud2[c]);
      }
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint32_t* us = us2[c];
        const uint32_t* ud = ud2[c];
        float p[32], ds[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(lse + 32 * c + i);
          const float4 d4 = *reinterpret_cast<const float4*>(dlt + 32 * c + i);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
          const float dl[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float pv = bwd_ex2(fmaf(__uint_as_float(us[i + e]), args.scale_log2, -lv[e]));
            p[i + e] = pv;
            ds[i + e] = pv * (__uint_as_float(ud[i + e]) - dl[e]) * args.scale;
          }
        }
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int qi = q0 + 32 * c + i;
            const bool m = (qi >= S) || (kj >= Sk) || (args.causal && kj > qi + qoff) || (qi >= qhi);
            p[i] = m ? 0.f : p[i];
            ds[i] = m ? 0.f : ds[i];
          }
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(p[2 * i], p[2 * i + 1]);
        // P^T as packed bf16 over S^T[w]: query column q lands in TMEM column q / 2
        // (this thread's own lane, already loaded, so no cross-thread hazard).
        tmem_st16(tS + 16 * c, pk);
        // dS^T row r, query columns [32c, 32c + 32): 128B-swizzled K-major tile
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          const int unit = (32 * c + i) >> 3;
          uint4 v;
          v.x = pack_bf16(ds[i + 0], ds[i + 1]);
          v.y = pack_bf16(ds[i + 2], ds[i + 3]);
          v.z = pack_bf16(ds[i + 4], ds[i + 5]);
          v.w = pack_bf16(ds[i + 6], ds[i + 7]);
          *reinterpret_cast<uint4*>(ds_tile + r * 128 + ((unit ^ (r & 7)) << 4)) = v;
        }
      }
      tmem_wait_st();
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pds_ready[w]);
      // dQ^T drain: thread = head dim r, 64 query columns -> fp32 staging in the
      // Q/dO stage of this iteration (once its dV / dK MMAs have released the
      // stage) as four 64-row x 32-column 128B-swizzled boxes; the lanes of a
      // warp write one 128-byte row per store.
      if (!mbar_wait(&dq_full[w], ph, err, kErrTimeoutSoftmax)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t u[2][32];
        tmem_ld32(tP, u[0]);
        tmem_ld32(tP + 32, u[1]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dq_free[w]);
        // dV / dK of this iteration may still read Q / dO from the stage
        if (!mbar_wait(&qdo_empty[s], static_cast<uint32_t>(it / PNS) & 1, err, kErrTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* box = (quarter < 2 ? sQ(s) : sDO(s)) + (quarter & 1) * (PBQ * 128);
        const int chunk = lane >> 2, sub = (lane & 3) * 4;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int q = 32 * c + i;
            *reinterpret_cast<uint32_t*>(box + q * 128 + ((chunk ^ (q & 7)) << 4) + sub) = u[c][i];
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&staged[s]);
      }
    }
    // ------------------------------------------------------- dK / dV out
    if (ok && n_iter > 0 && mbar_wait(acc_done, 0, err, kErrTimeoutSoftmax)) {
      tc_fence_after();
      const bool row_ok = kj < Sk;
      const bool cp = args.dkv_cp != nullptr;
      float* dk = cp ? args.dkv_cp + (static_cast<int64_t>(ktok0 + kj) * (2 * args.Hk) + hk) * D
                     : args.dqk + (static_cast<int64_t>(tok0 + kj) * (args.Hq + args.Hk) + args.Hq + hk) * D;
      float* dv_cp = cp ? args.dkv_cp + (static_cast<int64_t>(ktok0 + kj) * (2 * args.Hk) + args.Hk + hk) * D
                        : nullptr;
      __nv_bfloat16* dv = cp ? nullptr
                             : args.dqkv + (static_cast<int64_t>(tok0 + kj) * (args.Hq + 2 * args.Hk) + args.Hq + args.Hk + hk) * D;
#pragma unroll
      for (int c = 0; c < D / 2; c += 32) {
        const int cc = (D / 2) * w + c;
        uint32_t uk[32], uv[32];
        tmem_ld32(tDK + lane_base + cc, uk);
        tmem_ld32(tDV + lane_base + cc, uv);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dk + cc + i) = make_float4(__uint_as_float(uk[i]), __uint_as_float(uk[i + 1]),
                                                                __uint_as_float(uk[i + 2]), __uint_as_float(uk[i + 3]));
          if (cp) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dv_cp + cc + i) = make_float4(__uint_as_float(uv[i]), __uint_as_float(uv[i + 1]),
                                                                       __uint_as_float(uv[i + 2]), __uint_as_float(uv[i + 3]));
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 v;
              v.x = pack_bf16(__uint_as_float(uv[q * 8 + 0]), __uint_as_float(uv[q * 8 + 1]));
              v.y = pack_bf16(__uint_as_float(uv[q * 8 + 2]), __uint_as_float(uv[q * 8 + 3]));
              v.z = pack_bf16(__uint_as_float(uv[q * 8 + 4]), __uint_as_float(uv[q * 8 + 5]));
              v.w = pack_bf16(__uint_as_float(uv[q * 8 + 6]), __uint_as_float(uv[q * 8 + 7]));
              reinterpret_cast<uint4*>(dv + cc)[q] = v;
            }
          }
        }
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

// delta[b,h,q] = sum_d dO * O ; also zeroes the dq part of dqk.  D/8 lanes per
// (token, head) row, 16-byte loads, a shuffle reduction inside the lane group;
// every lane of a warp runs the same number of iterations (full-mask shuffles).
template <int D>
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* __restrict__ dO, const __nv_bfloat16* __restrict__ O,
                                    float* __restrict__ delta, float* __restrict__ dqk, int B, int S,
                                    int Hq, int Hk) {
  constexpr int G = D / 8;             // lanes per row
  constexpr int RPW = 32 / G;          // rows per warp and iteration
  const int lane = threadIdx.x & 31;
  const int sub = lane % G;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t items = static_cast<int64_t>(B) * S * Hq;
  for (int64_t base = gw * RPW; base < items; base += warps * RPW) {
    const int64_t it = base + lane / G;
    const bool ok = it < items;
    const int64_t t = ok ? it / Hq : 0;
    const int h = ok ? static_cast<int>(it - t * Hq) : 0;
    float x[8], y[8];
    float s = 0.f;
    if (ok) {
      load8(dO + (t * Hq + h) * D + sub * 8, x);
      load8(O + (t * Hq + h) * D + sub * 8, y);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += x[i] * y[i];
    }
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (ok) {
      const int b = static_cast<int>(t / S);
      const int q = static_cast<int>(t - static_cast<int64_t>(b) * S);
      if (sub == 0) delta[(static_cast<int64_t>(b) * Hq + h) * S + q] = s;
      float4* dq = reinterpret_cast<float4*>(dqk + (t * (Hq + Hk) + h) * D + sub * 8);
      dq[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      dq[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

struct AttnBwdKV {           // context parallelism (see AttnBwdArgs)
  const torch::Tensor* kv = nullptr;
  torch::Tensor* dkv = nullptr;
  int Sk = 0, off0 = 0, off1 = 0, split = 0;
  const int* q_hi = nullptr;  // key-range mask (self-attention only)
};

template <int D>
static torch::Tensor launch_attn_bwd(const torch::Tensor& dO, const torch::Tensor& qk, const torch::Tensor& qkv,
                                     const torch::Tensor& O, const torch::Tensor& lse, torch::Tensor& dqkv,
                                     int B, int S, int Hq, int Hk, bool causal, float scale,
                                     const AttnBwdKV& cp = AttnBwdKV()) {
  using L = AttnBwdSmem<D>;
  static_assert(L::kBytes <= 232448 && AttnBwdPPSmem::kBytes <= 232448, "attention backward shared memory budget");
  const int64_t T = static_cast<int64_t>(B) * S;
  auto dqk = torch::empty({T, (int64_t)(Hq + Hk) * D}, qk.options().dtype(torch::kFloat32));
  auto delta = torch::empty({B, Hq, S}, qk.options().dtype(torch::kFloat32));
  auto st = at::cuda::getCurrentCUDAStream();
  {
    const int64_t rows_per_block = 256 / (D / 8);
    const int64_t blocks = (T * Hq + rows_per_block - 1) / rows_per_block;
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, num_sms() * 8)));
    attn_bwd_pre_kernel<D><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(dO.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(O.data_ptr()),
        delta.data_ptr<float>(), dqk.data_ptr<float>(), B, S, Hq, Hk);
    NQ_CHECK_CUDA(cudaGetLastError());
  }
  // head_dim 128 runs the ping-pong kernel on 64-query tiles
  constexpr bool kPP = (D == 128);
  const int qrows = kPP ? PBQ : 128;
  auto tq = make_tmap_3d_bf16(qk.data_ptr(), D, Hq + Hk, T, D, (int64_t)(Hq + Hk) * D, 64, 1, qrows);
  auto tdo = make_tmap_3d_bf16(dO.data_ptr(), D, Hq, T, D, (int64_t)Hq * D, 64, 1, qrows);
  auto tdq = make_tmap_3d_f32(dqk.data_ptr(), D, Hq + Hk, T, D, (int64_t)(Hq + Hk) * D, 32, 1, qrows);
  CUtensorMap tv, tk;
  AttnBwdArgs a;
  if (cp.kv != nullptr) {
    const int64_t Tk = static_cast<int64_t>(B) * cp.Sk;
    tk = make_tmap_3d_bf16(cp.kv->data_ptr(), D, 2 * Hk, Tk, D, (int64_t)(2 * Hk) * D, 64, 1, 128);
    tv = tk;
    a.Sk = cp.Sk; a.k_head = 0; a.v_head = Hk;
    a.off0 = cp.off0; a.off1 = cp.off1; a.split = cp.split;
    a.dkv_cp = cp.dkv->data_ptr<float>();
  } else {
    tv = make_tmap_3d_bf16(qkv.data_ptr(), D, Hq + 2 * Hk, T, D, (int64_t)(Hq + 2 * Hk) * D, 64, 1, 128);
    tk = kPP ? make_tmap_3d_bf16(qk.data_ptr(), D, Hq + Hk, T, D, (int64_t)(Hq + Hk) * D, 64, 1, 128) : tq;
    a.Sk = S; a.k_head = Hq; a.v_head = Hq + Hk;
    a.off0 = 0; a.off1 = 0; a.split = S;
    a.dkv_cp = nullptr;
  }
  a.q_hi = cp.q_hi;
  a.B = B; a.S = S; a.Hq = Hq; a.Hk = Hk;
  a.scale = scale;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal = causal ? 1 : 0;
  a.lse = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.dqk = dqk.data_ptr<float>();
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.err = error_flag_ptr();
  auto kern = attn_bwd_pp_kernel;
  int bytes = AttnBwdPPSmem::kBytes;
  if constexpr (!kPP) {
    kern = attn_bwd_kernel<D>;
    bytes = L::kBytes;
  }
  set_max_smem_once(reinterpret_cast<const void*>(kern), bytes);
  const int grid = B * Hk * ((a.Sk + BKN - 1) / BKN);
  kern<<<grid, kBwdThreads, bytes, st>>>(tq, tv, tdo, tdq, tk, a);
  NQ_CHECK_CUDA(cudaGetLastError());
  return dqk;
}

// Returns dq|dk fp32 [T, (Hq+Hk)*D]; writes dv (bf16) into the v slot of dqkv.
torch::Tensor attn_bwd(torch::Tensor dO, torch::Tensor qk, torch::Tensor qkv, torch::Tensor O,
                       torch::Tensor lse, torch::Tensor dqkv, int64_t B, int64_t S, int64_t Hq,
                       int64_t Hk, int64_t D, bool causal, double scale, c10::optional<torch::Tensor> q_hi) {
  check_bf16(dO, "dO"); check_bf16(qk, "qk"); check_bf16(qkv, "qkv"); check_bf16(O, "O"); check_bf16(dqkv, "dqkv");
  TORCH_CHECK(dO.is_contiguous() && O.is_contiguous() && dqkv.is_contiguous(), "attn_bwd: contiguous");
  c10::cuda::CUDAGuard g(qk.device());
  AttnBwdKV self;
  if (q_hi.has_value() && q_hi->defined()) {
    TORCH_CHECK(causal, "attn_bwd: the key-range mask applies to causal attention");
    TORCH_CHECK(q_hi->is_cuda() && q_hi->scalar_type() == torch::kInt32 && q_hi->is_contiguous() &&
                    q_hi->numel() == B * S, "attn_bwd: q_hi int32 [B*S]");
    self.q_hi = q_hi->data_ptr<int>();
  }
  if (D == 128) return launch_attn_bwd<128>(dO, qk, qkv, O, lse, dqkv, B, S, Hq, Hk, causal, (float)scale, self);
  if (D == 64) return launch_attn_bwd<64>(dO, qk, qkv, O, lse, dqkv, B, S, Hq, Hk, causal, (float)scale, self);
  TORCH_CHECK(false, "attn_bwd: head_dim must be 64 or 128");
  return torch::Tensor();
}

// Context-parallel backward (see attn_fwd_cp): returns dq (and an unused dk
// slot) fp32 [B*S, (Hq+Hk)*D] for the local queries and dkv fp32
// [B*Sk, 2*Hk*D], this rank's partial gradient of the gathered keys/values.
std::vector<torch::Tensor> attn_bwd_cp(torch::Tensor dO, torch::Tensor qk, torch::Tensor kv, torch::Tensor O,
                                       torch::Tensor lse, int64_t B, int64_t S, int64_t Sk, int64_t Hq,
                                       int64_t Hk, int64_t D, int64_t off0, int64_t off1, int64_t split,
                                       double scale, c10::optional<torch::Tensor> dkv_out) {
  check_bf16(dO, "dO"); check_bf16(qk, "qk"); check_bf16(kv, "kv"); check_bf16(O, "O");
  TORCH_CHECK(dO.is_contiguous() && O.is_contiguous() && qk.is_contiguous() && kv.is_contiguous(),
              "attn_bwd_cp: contiguous");
  TORCH_CHECK(kv.size(0) == B * Sk && kv.size(1) == 2 * Hk * D, "attn_bwd_cp: kv shape");
  TORCH_CHECK(split % BQM == 0 && S % BQM == 0, "attn_bwd_cp: chunk lengths must be multiples of 128");
  c10::cuda::CUDAGuard g(qk.device());
  // key blocks no local query can see keep zero gradients
  torch::Tensor dkv;
  if (dkv_out.has_value() && dkv_out->defined()) {
    dkv = *dkv_out;
    TORCH_CHECK(dkv.scalar_type() == torch::kFloat32 && dkv.is_contiguous() && dkv.numel() == B * Sk * 2 * Hk * D,
                "attn_bwd_cp: dkv_out fp32 [B*Sk, 2*Hk*D]");
    dkv.zero_();
  } else {
    dkv = torch::zeros({B * Sk, 2 * Hk * D}, qk.options().dtype(torch::kFloat32));
  }
  AttnBwdKV cp;
  cp.kv = &kv; cp.dkv = &dkv; cp.Sk = static_cast<int>(Sk); cp.off0 = static_cast<int>(off0);
  cp.off1 = static_cast<int>(off1 - split);
  cp.split = static_cast<int>(split);
  torch::Tensor dummy_qkv = qk;  // unused V source in this mode
  torch::Tensor dq;
  if (D == 128) dq = launch_attn_bwd<128>(dO, qk, qk, O, lse, dummy_qkv, B, S, Hq, Hk, true, (float)scale, cp);
  else if (D == 64) dq = launch_attn_bwd<64>(dO, qk, qk, O, lse, dummy_qkv, B, S, Hq, Hk, true, (float)scale, cp);
  else TORCH_CHECK(false, "attn_bwd_cp: head_dim must be 64 or 128");
  return {dq, dkv};
}

}  // namespace nq
