// Persistent warp-specialised bf16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   C[M,N] = A * B^T with A, B either K-major or MN-major in global memory:
//     fwd    : A = X  [M,K] (K-major),   B = W [N,K] (K-major)      -> C bf16
//     dgrad  : A = dY [M,N'] (K-major),  B = W [N',K'] (MN-major)   -> C bf16
//     wgrad  : A = dY [T,N'] (MN-major), B = X [T,K'] (MN-major)    -> C fp32 +=
//   and grouped (mixture-of-experts) variants where groups split M (one
//   weight per group) or K (one fp32 output per group).
//
// CTA = 6 warps: warp 0 issues TMA loads into a STAGES-deep shared-memory ring,
// warp 1 (one elected thread) issues tcgen05.mma 128xBNx16 into one of two TMEM
// accumulators, warps 2-5 drain the other accumulator (tcgen05.ld -> registers
// -> global) so the epilogue of tile i overlaps the main loop of tile i+1.  One
// CTA per SM walks the tile list with a grid stride; tiles are rasterised in
// bands of 8 M-tiles for L2 reuse of B.
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"
#include "peer.cuh"
#include "tmap.h"

namespace nq {

constexpr int GBM = 128;
constexpr int GBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kMaxGroups = 256;

enum GroupMode : int { kGroupNone = 0, kGroupM = 1, kGroupK = 2 };
// kEpiSwiGLU: B = [gate; up] rows [2I, K]; tile n covers gate rows
// [128n, 128n+128) and the matching up rows (two 128-row TMA boxes stacked in
// the B stage), so one accumulator holds g and u of the same 128 intermediate
// columns.  The epilogue stores gu = [g | u] (bf16, kept for the backward) and
// h = silu(g) * u computed from the bf16-rounded g, u (what a separate SwiGLU
// pass over gu would produce).
enum EpiMode : int { kEpiBF16 = 0, kEpiAccF32 = 1, kEpiSwiGLU = 2 };

struct GemmArgs {
  int M, N, K;
  void* C;
  int64_t ldc;
  int group_mode;
  int num_groups;
  const int* offsets;       // [num_groups+1], rows (group M) or k-rows (group K)
  int64_t c_group_stride;   // group K: elements between the groups' outputs
  int b_group_rows;         // group M: rows of B per group in the tensor map's row space
  int* err;
  __nv_bfloat16* H;          // kEpiSwiGLU: h [M, N/2]
  int64_t ldh;
  // Tensor-parallel all-gather consumer (peer.cuh protocol): before loading the
  // first A tile of an m-tile, wait until ag_flags[row owner] reaches ag_seq.
  const unsigned* ag_flags;  // null: no wait
  unsigned ag_seq;
  int tp_rows;               // rows per rank: owner = row / tp_rows
  // Tensor-parallel reduce-scatter epilogue: a finished row tile is stored into
  // rs_dst[owner] at the owner-local row; the last CTA publishes rs_seq into
  // every rank's flag block at rs_flag_idx.
  int rs;
  int tp_world;
  __nv_bfloat16* rs_dst[8];
  unsigned* rs_flag_dst[8];
  int rs_flag_idx;
  unsigned rs_seq;
  unsigned* rs_counter;
  unsigned rs_target;
  // 1: the epilogue writes C (and H) through shared memory with TMA stores
  // (bf16) or TMA add-reductions (fp32 accumulate) using the tmC / tmH maps
  // (box 32 x 32 rows).  0: register-to-global stores.
  int tma_epi;
  // Expert-parallel consumer (group M): the A rows of local expert g's
  // segment arrive from the source ranks in rank order, source s holding
  // ep_counts[s * ep_E + ep_expert0 + g] rows.  Before loading an m-tile the
  // producer waits for the dispatch flag ep_flags[s] >= ep_seq of every
  // source whose rows the tile covers, so tiles start as their rows land.
  const int* ep_counts;      // null: no wait
  const unsigned* ep_flags;
  unsigned ep_seq;
  int ep_world, ep_E, ep_expert0;
};

// Epilogue staging for TMA stores: per epilogue warp (32 rows) three 2 KB
// boxes of 32 rows x 64 B (bf16: 32 columns; SwiGLU: g, u and h), or one
// 4 KB box of 32 rows x 32 fp32 columns.  Rows are dense (no swizzle); each
// lane writes its row's 16-byte pieces in a lane-rotated order, so a warp's
// shared-memory stores are free of bank conflicts.
constexpr int kEpiWarpBytes = 6144;

// Reduce-scatter destinations as tensor maps (one per owner rank): the
// tensor-parallel epilogue writes each finished row tile into its owner's
// partial buffer with TMA stores (64-byte row pieces) instead of 16-byte
// register stores across NVLink.  Plain stores, no multicast.
struct RsMaps {
  CUtensorMap m[8];
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = GBM * GBK * 2;
  static constexpr int kBBytes = BN * GBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOff = STAGES * kStageBytes;
  static constexpr int kEpiOff = (kBarOff + 1024 + 4 * (kMaxGroups + 1) + 1023) / 1024 * 1024;
  static constexpr int kBytes = kEpiOff + 4 * kEpiWarpBytes + 1024;  // + align slack
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mt, int& nt) {
  const int band_tiles = 8 * tiles_n;
  const int band = t / band_tiles;
  const int r = t - band * band_tiles;
  const int m_base = band * 8;
  const int bm = min(8, tiles_m - m_base);
  mt = m_base + r % bm;
  nt = r / bm;
}

// TMA-store epilogue of one accumulator tile for one epilogue warp: rows
// [ty, ty+32) of C, columns [n0, n0+BN) read from TMEM at `trow` (the warp's
// lane quarter, the tile's accumulator buffer); `stg` is the warp's staging.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tma(uint8_t* stg, uint32_t trow, int ty, int n0, const GemmArgs& args,
                                             const CUtensorMap* tmC, const CUtensorMap* tmH, bool has_acc,
                                             int lane, int& half) {
  if (EPI == kEpiSwiGLU) {
    const int I = args.N >> 1;
#pragma unroll 1
    for (int c = 0; c < BN / 2; c += 32) {
      uint32_t rg[32], ru[32];
      tmem_ld32(trow + c, rg);
      tmem_ld32(trow + BN / 2 + c, ru);
      tmem_wait_ld();
      const int jc = n0 / 2 + c;
      if (jc >= I) continue;
      uint4 vg[4], vu[4], vh[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float g[8], u[8], h[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          g[e] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rg[q * 8 + e])));
          u[e] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(ru[q * 8 + e])));
          h[e] = g[e] * sigmoid_fast(g[e]) * u[e];
        }
        vg[q] = make_uint4(pack_bf16(g[0], g[1]), pack_bf16(g[2], g[3]), pack_bf16(g[4], g[5]),
                           pack_bf16(g[6], g[7]));
        vu[q] = make_uint4(pack_bf16(u[0], u[1]), pack_bf16(u[2], u[3]), pack_bf16(u[4], u[5]),
                           pack_bf16(u[6], u[7]));
        vh[q] = make_uint4(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]), pack_bf16(h[4], h[5]),
                           pack_bf16(h[6], h[7]));
      }
      if (lane == 0) bulk_wait_read_all();  // the previous chunk's stores have read the staging
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int q = (j + lane) & 3;
        const uint4 a = q == 0 ? vg[0] : q == 1 ? vg[1] : q == 2 ? vg[2] : vg[3];
        const uint4 b = q == 0 ? vu[0] : q == 1 ? vu[1] : q == 2 ? vu[2] : vu[3];
        const uint4 d = q == 0 ? vh[0] : q == 1 ? vh[1] : q == 2 ? vh[2] : vh[3];
        *reinterpret_cast<uint4*>(stg + lane * 64 + q * 16) = a;
        *reinterpret_cast<uint4*>(stg + 2048 + lane * 64 + q * 16) = b;
        *reinterpret_cast<uint4*>(stg + 4096 + lane * 64 + q * 16) = d;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmC, stg, jc, ty);
        tma_store_2d(tmC, stg + 2048, I + jc, ty);
        tma_store_2d(tmH, stg + 4096, jc, ty);
        bulk_commit();
      }
    }
  } else if (EPI == kEpiBF16 && has_acc) {
    // `half` alternates the two staging halves across chunks and tiles, so
    // the store still in flight always reads the other half
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(trow + c, r);
      tmem_wait_ld();
      if (n0 + c >= args.N) continue;
      uint4 v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        v[q] = make_uint4(pack_bf16(__uint_as_float(r[q * 8 + 0]), __uint_as_float(r[q * 8 + 1])),
                          pack_bf16(__uint_as_float(r[q * 8 + 2]), __uint_as_float(r[q * 8 + 3])),
                          pack_bf16(__uint_as_float(r[q * 8 + 4]), __uint_as_float(r[q * 8 + 5])),
                          pack_bf16(__uint_as_float(r[q * 8 + 6]), __uint_as_float(r[q * 8 + 7])));
      uint8_t* dst = stg + half * 2048;
      if (lane == 0) bulk_wait_read_1();  // the store that last read this half is done reading
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int q = (j + lane) & 3;
        *reinterpret_cast<uint4*>(dst + lane * 64 + q * 16) = q == 0 ? v[0] : q == 1 ? v[1] : q == 2 ? v[2] : v[3];
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmC, dst, n0 + c, ty);
        bulk_commit();
      }
      half ^= 1;
    }
  } else if (EPI == kEpiAccF32 && has_acc) {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(trow + c, r);
      tmem_wait_ld();
      if (n0 + c >= args.N) continue;
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = (j + lane) & 7;
        uint4 v = make_uint4(r[0], r[1], r[2], r[3]);
#pragma unroll
        for (int t = 1; t < 8; ++t)
          if (q == t) v = make_uint4(r[4 * t], r[4 * t + 1], r[4 * t + 2], r[4 * t + 3]);
        *reinterpret_cast<uint4*>(stg + lane * 128 + q * 16) = v;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d(tmC, stg, n0 + c, ty);
        bulk_commit();
      }
    }
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmH,
                const __grid_constant__ RsMaps rsm, const GemmArgs args) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* s_off = reinterpret_cast<int*>(smem + L::kBarOff + 1024);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = args.err;

  const int tiles_n = (args.N + BN - 1) / BN;
  int tiles_m, total_tiles;
  if (args.group_mode == kGroupM) {
    tiles_m = 0;  // computed below from offsets
  }
  if (args.group_mode != kGroupNone) {
    for (int i = threadIdx.x; i <= args.num_groups; i += blockDim.x) s_off[i] = args.offsets[i];
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.tma_epi) {
      tma_prefetch_desc(&tmC);
      if (EPI == kEpiSwiGLU) tma_prefetch_desc(&tmH);
    }
  }
  constexpr uint32_t kTmemCols = (2 * BN <= 32) ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (args.group_mode == kGroupM) {
    tiles_m = s_off[args.num_groups] / GBM;
    total_tiles = tiles_m * tiles_n;
  } else if (args.group_mode == kGroupK) {
    tiles_m = (args.M + GBM - 1) / GBM;
    total_tiles = args.num_groups * tiles_m * tiles_n;
  } else {
    tiles_m = (args.M + GBM - 1) / GBM;
    total_tiles = tiles_m * tiles_n;
  }
  const int per_group = tiles_m * tiles_n;

  // Decode tile t -> (m0, n0, group, k range in elements).
  auto decode = [&](int t, int& m0, int& n0, int& g, int& kb, int& ke) {
    int tt = t;
    g = 0;
    if (args.group_mode == kGroupK) {
      g = t / per_group;
      tt = t - g * per_group;
    }
    int mt, nt;
    tile_coords(tt, tiles_m, tiles_n, mt, nt);
    m0 = mt * GBM;
    n0 = nt * BN;
    if (args.group_mode == kGroupM) {
      int lo = 0, hi = args.num_groups - 1;
      while (lo < hi) {  // last group with s_off[g] <= m0
        int mid = (lo + hi + 1) >> 1;
        if (s_off[mid] <= m0) lo = mid; else hi = mid - 1;
      }
      g = lo;
    }
    if (args.group_mode == kGroupK) {
      kb = s_off[g];
      ke = s_off[g + 1];
    } else {
      kb = 0;
      ke = args.K;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int waited_owner = -1;
      unsigned waited_src = 0;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        int m0, n0, g, kb, ke;
        decode(t, m0, n0, g, kb, ke);
        const int b_row_off = (args.group_mode == kGroupM) ? g * args.b_group_rows : 0;
        if (args.ep_counts != nullptr && args.group_mode == kGroupM) {
          const int e = args.ep_expert0 + g;
          const int r0 = m0 - s_off[g];
          int pre = 0;
          for (int src = 0; src < args.ep_world; ++src) {
            const int c = args.ep_counts[src * args.ep_E + e];
            if (c > 0 && pre < r0 + GBM && pre + c > r0 && !((waited_src >> src) & 1u)) {
              if (!wait_flag(args.ep_flags + src, args.ep_seq, err)) { ok = false; break; }
              waited_src |= 1u << src;
              asm volatile("fence.proxy.async.global;" ::: "memory");
            }
            pre += c;
          }
          if (!ok) break;
        }
        if (args.ag_flags != nullptr) {
          const int owner = m0 / args.tp_rows;
          if (owner != waited_owner) {
            if (!wait_flag(args.ag_flags + owner, args.ag_seq, err)) { ok = false; break; }
            // peers wrote these rows with generic stores; TMA reads via the async proxy
            asm volatile("fence.proxy.async.global;" ::: "memory");
            waited_owner = owner;
          }
        }
        for (int k0 = kb; k0 < ke; k0 += GBK) {
          if (!mbar_wait(&empty[stage], phase ^ 1, err, kErrTimeoutProducer)) { ok = false; break; }
          uint8_t* sA = smem + stage * L::kStageBytes;
          uint8_t* sB = sA + L::kABytes;
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          if (!A_MN) {
            tma_load_2d(sA, &tmA, &full[stage], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < GBM / 64; ++j) tma_load_2d(sA + j * 8192, &tmA, &full[stage], m0 + 64 * j, k0);
          }
          if (EPI == kEpiSwiGLU) {
            tma_load_2d(sB, &tmB, &full[stage], k0, n0 / 2);                         // gate rows
            tma_load_2d(sB + 128 * GBK * 2, &tmB, &full[stage], k0, args.N / 2 + n0 / 2);  // up rows
          } else if (!B_MN) {
            tma_load_2d(sB, &tmB, &full[stage], k0, b_row_off + n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sB + j * 8192, &tmB, &full[stage], n0 + 64 * j, b_row_off + k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: wait (bounded) until every issued load has landed before exiting.
      if (!ok) {
        for (int s = 0; s < STAGES; ++s) {
          uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&full[s], 0) && !mbar_try_wait(&full[s], 1)) {
            if (globaltimer() - t0 > 100000000ull) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_bf16(GBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++local) {
        int m0, n0, g, kb, ke;
        decode(t, m0, n0, g, kb, ke);
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        uint32_t acc = 0;
        for (int k0 = kb; k0 < ke; k0 += GBK) {
          if (!mbar_wait(&full[stage], phase, err, kErrTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < GBK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_addr + kk * 2048, 8192, 1024)
                                     : sdesc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_addr + kk * 2048, 8192, 1024)
                                     : sdesc_sw128(b_addr + kk * 32, 16, 1024);
            umma_bf16(d_tmem, ad, bd, idesc, acc);
            acc = 1;
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (acc) umma_commit(&tfull[buf]);
        else mbar_arrive(&tfull[buf]);  // empty K range: nothing accumulated
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    int stg_half = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++local) {
      int m0, n0, g, kb, ke;
      decode(t, m0, n0, g, kb, ke);
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&tfull[buf], use & 1, err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const int m_limit = (args.group_mode == kGroupM) ? s_off[args.num_groups] : args.M;
      const bool row_ok = row < m_limit;
      const bool has_acc = ke > kb;
      if (args.tma_epi && args.rs) {
        // reduce-scatter: the tile's rows belong to one owner (tp_rows % 128 == 0)
        const int owner = m0 / args.tp_rows;
        epilogue_tma<BN, EPI>(smem + L::kEpiOff + quarter * kEpiWarpBytes,
                              tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN,
                              m0 - owner * args.tp_rows + quarter * 32, n0, args, &rsm.m[owner], &tmH,
                              has_acc, lane, stg_half);
      } else if (args.tma_epi) {
        epilogue_tma<BN, EPI>(smem + L::kEpiOff + quarter * kEpiWarpBytes,
                              tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN,
                              m0 + quarter * 32, n0, args, &tmC, &tmH, has_acc, lane, stg_half);
      } else if (EPI == kEpiSwiGLU) {
        const int I = args.N >> 1;
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          uint32_t rg[32], ru[32];
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN + c;
          tmem_ld32(taddr, rg);
          tmem_ld32(taddr + BN / 2, ru);
          tmem_wait_ld();
          const int jc = n0 / 2 + c;
          if (!row_ok || jc >= I) continue;
          __nv_bfloat16* G = reinterpret_cast<__nv_bfloat16*>(args.C) + static_cast<int64_t>(row) * args.ldc + jc;
          __nv_bfloat16* Hp = args.H + static_cast<int64_t>(row) * args.ldh + jc;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float g[8], u[8], h[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              g[e] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rg[q * 8 + e])));
              u[e] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(ru[q * 8 + e])));
              const float sg = sigmoid_fast(g[e]);
              h[e] = g[e] * sg * u[e];
            }
            reinterpret_cast<uint4*>(G)[q] = make_uint4(pack_bf16(g[0], g[1]), pack_bf16(g[2], g[3]),
                                                        pack_bf16(g[4], g[5]), pack_bf16(g[6], g[7]));
            reinterpret_cast<uint4*>(G + I)[q] = make_uint4(pack_bf16(u[0], u[1]), pack_bf16(u[2], u[3]),
                                                            pack_bf16(u[4], u[5]), pack_bf16(u[6], u[7]));
            reinterpret_cast<uint4*>(Hp)[q] = make_uint4(pack_bf16(h[0], h[1]), pack_bf16(h[2], h[3]),
                                                         pack_bf16(h[4], h[5]), pack_bf16(h[6], h[7]));
          }
        }
      } else if (has_acc) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN + c, r);
          tmem_wait_ld();
          const int col = n0 + c;
          if (!row_ok || col >= args.N) continue;
          const int ncols = min(32, args.N - col);
          if (EPI == kEpiBF16) {
            __nv_bfloat16* Cp;
            if (args.rs) {
              const int owner = row / args.tp_rows;
              Cp = args.rs_dst[owner] + static_cast<int64_t>(row - owner * args.tp_rows) * args.ldc + col;
            } else {
              Cp = reinterpret_cast<__nv_bfloat16*>(args.C) + static_cast<int64_t>(row) * args.ldc + col;
            }
            if (ncols == 32 && (reinterpret_cast<uintptr_t>(Cp) & 15) == 0) {
              uint4* dst = reinterpret_cast<uint4*>(Cp);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 v;
                v.x = pack_bf16(__uint_as_float(r[q * 8 + 0]), __uint_as_float(r[q * 8 + 1]));
                v.y = pack_bf16(__uint_as_float(r[q * 8 + 2]), __uint_as_float(r[q * 8 + 3]));
                v.z = pack_bf16(__uint_as_float(r[q * 8 + 4]), __uint_as_float(r[q * 8 + 5]));
                v.w = pack_bf16(__uint_as_float(r[q * 8 + 6]), __uint_as_float(r[q * 8 + 7]));
                dst[q] = v;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncols) Cp[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
            }
          } else {
            float* Cp = reinterpret_cast<float*>(args.C) + static_cast<int64_t>(g) * args.c_group_stride +
                        static_cast<int64_t>(row) * args.ldc + col;
            if (ncols == 32 && (reinterpret_cast<uintptr_t>(Cp) & 15) == 0) {
              float4* p4 = reinterpret_cast<float4*>(Cp);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 v = p4[q];
                v.x += __uint_as_float(r[q * 4 + 0]);
                v.y += __uint_as_float(r[q * 4 + 1]);
                v.z += __uint_as_float(r[q * 4 + 2]);
                v.w += __uint_as_float(r[q * 4 + 3]);
                p4[q] = v;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncols) Cp[j] += __uint_as_float(r[j]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    // TMA stores complete before the CTA's shared memory goes away (and, for
    // the reduce-scatter, before the grid's completion flag is published)
    if (args.tma_epi && lane == 0) {
      bulk_wait_all();
      if (args.rs) asm volatile("fence.proxy.async.global;" ::: "memory");
    }
  }

  tc_fence_before();
  __syncthreads();
  if (args.rs)
    grid_done_signal(args.rs_counter, args.rs_target, args.rs_flag_dst, args.rs_flag_idx,
                     args.tp_world, args.rs_seq);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------- 2-SM (CTA pair)
// Same GEMMs on CTA pairs: a cluster of two CTAs computes a 256 x 256 output
// tile with tcgen05.mma.cta_group::2 (M = 256: 128 rows per CTA; B: each CTA
// stages 128 of the 256 columns).  Per k-block each SM loads 32 KB (its A rows
// and its half of B) instead of 48 KB for a 128 x 256 tile on one SM, so a
// FLOP costs a third less L2-to-shared traffic and shared-memory bandwidth.
//   warp 0 (both CTAs)  : TMA loads into its own ring; completion bytes count
//                          on the even CTA's `full` barrier;
//   warp 1 (even CTA)   : waits `full`, issues the pair MMAs, commits stage
//                          release and accumulator-ready to both CTAs;
//   warps 2-5 (both)    : drain the CTA's 128 accumulator rows with the TMA
//                          epilogue, then arrive on the even CTA's `tempty`.
// No TMA multicast is used (loads read global memory of this GPU only, but
// the kernel is meant for multi-GPU jobs too).
constexpr int kPairStages = 6;

struct GemmPairSmem {
  static constexpr int kABytes = 128 * GBK * 2;   // this CTA's 128 rows of A
  static constexpr int kBBytes = 128 * GBK * 2;   // this CTA's 128 columns of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOff = kPairStages * kStageBytes;
  static constexpr int kEpiOff = kBarOff + 1024;
  static constexpr int kBytes = kEpiOff + 4 * kEpiWarpBytes + 1024;
};

template <bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1) __cluster_dims__(2, 1, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmH,
                     const GemmArgs args) {
  using L = GemmPairSmem;
  constexpr int STAGES = kPairStages;
  constexpr int BN = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const bool leader = cta == 0;
  int* err = args.err;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // 4 epilogue warps x 2 CTAs
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    if (EPI == kEpiSwiGLU) tma_prefetch_desc(&tmH);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  // the peer's loads and arrivals target this CTA's barriers: both CTAs'
  // barriers are initialised before anyone proceeds
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_m = (args.M + 255) / 256;
  const int tiles_n = (args.N + BN - 1) / BN;
  const int total = tiles_m * tiles_n;
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += pairs) {
        int mt, nt;
        tile_coords(t, tiles_m, tiles_n, mt, nt);
        const int m0 = mt * 256 + 128 * static_cast<int>(cta);  // this CTA's A rows
        const int n0 = nt * BN;
        for (int k0 = 0; k0 < args.K; k0 += GBK) {
          if (!mbar_wait(&empty[stage], phase ^ 1, err, kErrTimeoutProducer)) { ok = false; break; }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          uint8_t* sA = smem + stage * L::kStageBytes;
          uint8_t* sB = sA + L::kABytes;
          if (!A_MN) {
            tma_load_2d_pair(sA, &tmA, bar, k0, m0);
          } else {
            tma_load_2d_pair(sA, &tmA, bar, m0, k0);
            tma_load_2d_pair(sA + 8192, &tmA, bar, m0 + 64, k0);
          }
          if (EPI == kEpiSwiGLU) {
            // even CTA: the gate rows of this tile, odd CTA: the matching up rows
            tma_load_2d_pair(sB, &tmB, bar, k0, (cta ? args.N / 2 : 0) + n0 / 2);
          } else if (!B_MN) {
            tma_load_2d_pair(sB, &tmB, bar, k0, n0 + 128 * static_cast<int>(cta));
          } else {
            tma_load_2d_pair(sB, &tmB, bar, n0 + 128 * static_cast<int>(cta), k0);
            tma_load_2d_pair(sB + 8192, &tmB, bar, n0 + 128 * static_cast<int>(cta) + 64, k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {  // let loads already issued land before the CTA can exit
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 200000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------- MMA issuer (even CTA only)
    if (leader && elect_one()) {
      constexpr uint32_t idesc = idesc_bf16(256, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += pairs, ++local) {
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(&tempty[buf], (use & 1) ^ 1, err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        uint32_t acc = 0;
        for (int k0 = 0; k0 < args.K; k0 += GBK) {
          if (!mbar_wait(&full[stage], phase, err, kErrTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < GBK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_addr + kk * 2048, 8192, 1024)
                                     : sdesc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_addr + kk * 2048, 8192, 1024)
                                     : sdesc_sw128(b_addr + kk * 32, 16, 1024);
            umma_bf16_pair(d_tmem, ad, bd, idesc, acc);
            acc = 1;
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[buf], 0x3);
      }
    }
  } else {
    // ------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    int local = 0;
    int stg_half = 0;
    for (int t = pair; t < total; t += pairs, ++local) {
      int mt, nt;
      tile_coords(t, tiles_m, tiles_n, mt, nt);
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&tfull[buf], use & 1, err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      epilogue_tma<BN, EPI>(smem + L::kEpiOff + quarter * kEpiWarpBytes,
                            tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN,
                            mt * 256 + 128 * static_cast<int>(cta) + quarter * 32, nt * BN, args, &tmC, &tmH,
                            args.K > 0, lane, stg_half);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[buf]), 0));
    }
    if (lane == 0) bulk_wait_all();
  }

  // neither CTA leaves while the other may still signal its barriers or read
  // its shared memory / TMEM
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

// ----------------------------------------------------------------------- host
template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                        int max_tiles, cudaStream_t stream, const CUtensorMap* tc = nullptr,
                        const CUtensorMap* th = nullptr, const RsMaps* rsm = nullptr) {
  using L = GemmSmem<BN, STAGES>;
  static_assert(L::kBytes <= 232448, "GEMM shared memory budget");
  auto kern = gemm_kernel<BN, STAGES, A_MN, B_MN, EPI>;
  set_max_smem_once(reinterpret_cast<const void*>(kern), L::kBytes);
  int grid = std::min(num_sms(), std::max(1, max_tiles));
  CUtensorMap none;
  std::memset(&none, 0, sizeof(none));
  RsMaps no_rs;
  std::memset(&no_rs, 0, sizeof(no_rs));
  kern<<<grid, kGemmThreads, L::kBytes, stream>>>(ta, tb, tc ? *tc : none, th ? *th : none,
                                                  rsm ? *rsm : no_rs, a);
  NQ_CHECK_CUDA(cudaGetLastError());
}

// CTA-pair GEMM (the default where it applies: TMA epilogue usable and at
// least one tile per SM pair); NQ_GEMM_PAIR=0 in the environment, or
// gemm_pair_mode(0), selects the one-SM kernel everywhere.
static std::atomic<int> g_pair_mode{-1};

static bool pair_enabled() {
  int m = g_pair_mode.load(std::memory_order_relaxed);
  if (m < 0) {
    const char* e = std::getenv("NQ_GEMM_PAIR");
    m = (e == nullptr || std::string(e) != "0") ? 1 : 0;
    g_pair_mode.store(m, std::memory_order_relaxed);
  }
  return m != 0;
}

// mode 0 / 1 switches the CTA-pair kernels off / on; returns the mode before
// the call (a negative mode only queries it).
int64_t gemm_pair_mode(int64_t mode) {
  const int before = pair_enabled() ? 1 : 0;
  if (mode >= 0) g_pair_mode.store(mode ? 1 : 0, std::memory_order_relaxed);
  return before;
}

static bool rs_tma_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("NQ_RS_TMA");
    return e != nullptr && std::string(e) == "1";
  }();
  return on;
}

static bool use_pair(int M, int N) {
  return pair_enabled() && static_cast<int64_t>((M + 255) / 256) * ((N + 255) / 256) >= num_sms() / 2;
}

template <bool A_MN, bool B_MN, int EPI>
static void launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                             const CUtensorMap* th, const GemmArgs& a, cudaStream_t stream) {
  static_assert(GemmPairSmem::kBytes <= 232448, "pair GEMM shared memory budget");
  auto kern = gemm_pair_kernel<A_MN, B_MN, EPI>;
  set_max_smem_once(reinterpret_cast<const void*>(kern), GemmPairSmem::kBytes);
  const int tiles = ((a.M + 255) / 256) * ((a.N + 255) / 256);
  const int grid = 2 * std::max(1, std::min(num_sms() / 2, tiles));
  CUtensorMap none;
  std::memset(&none, 0, sizeof(none));
  kern<<<grid, kGemmThreads, GemmPairSmem::kBytes, stream>>>(ta, tb, tc, th ? *th : none, a);
  NQ_CHECK_CUDA(cudaGetLastError());
}

// TMA-store epilogue maps: C (bf16 or fp32) in 32 x 32 boxes, when its base
// and row stride meet TMA's 16-byte rules.
static bool tma_epi_ok(const void* p, int64_t ld, int elem) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (ld * elem) % 16 == 0;
}

constexpr int kBN = 256;
constexpr int kStages = 4;

static GemmArgs base_args(int M, int N, int K, void* C, int64_t ldc) {
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.C = C; a.ldc = ldc;
  a.group_mode = kGroupNone; a.num_groups = 1; a.offsets = nullptr;
  a.c_group_stride = 0; a.b_group_rows = 0; a.err = error_flag_ptr();
  a.tma_epi = 0;
  a.ep_counts = nullptr; a.ep_flags = nullptr; a.ep_seq = 0; a.ep_world = 0; a.ep_E = 0; a.ep_expert0 = 0;
  return a;
}

static inline int cdiv(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// C[M,N] (bf16) = A[M,K] @ B[N,K]^T
void gemm_nt_out(torch::Tensor A, torch::Tensor B, torch::Tensor C) {
  check_bf16(A, "A"); check_bf16(B, "B"); check_bf16(C, "C");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_nt: shape mismatch");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm_nt: inner dim must be contiguous");
  const int M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(C.size(0) == M && C.size(1) == N, "gemm_nt: C shape");
  if (M == 0 || N == 0) return;
  if (K == 0) { C.zero_(); return; }
  c10::cuda::CUDAGuard g(A.device());
  auto ta = make_tmap_2d_bf16(A.data_ptr(), M, K, A.stride(0), 64, GBM);
  auto a = base_args(M, N, K, C.data_ptr(), C.stride(0));
  CUtensorMap tc;
  if (tma_epi_ok(C.data_ptr(), C.stride(0), 2)) {
    tc = make_tmap_2d_bf16(C.data_ptr(), M, N, C.stride(0), 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    a.tma_epi = 1;
  }
  auto st = at::cuda::getCurrentCUDAStream();
  if (a.tma_epi && use_pair(M, N)) {
    auto tb = make_tmap_2d_bf16(B.data_ptr(), N, K, B.stride(0), 64, 128);
    launch_gemm_pair<false, false, kEpiBF16>(ta, tb, tc, nullptr, a, st);
    return;
  }
  auto tb = make_tmap_2d_bf16(B.data_ptr(), N, K, B.stride(0), 64, kBN);
  launch_gemm<kBN, kStages, false, false, kEpiBF16>(ta, tb, a, cdiv(M, GBM) * cdiv(N, kBN), st,
                                                    a.tma_epi ? &tc : nullptr);
}

torch::Tensor gemm_nt(torch::Tensor A, torch::Tensor B) {
  auto C = torch::empty({A.size(0), B.size(0)}, A.options());
  gemm_nt_out(A, B, C);
  return C;
}

// gu[M, 2I] = A[M,K] @ [gate; up]^T and h[M, I] = silu(gu[:, :I]) * gu[:, I:]
// in one GEMM (kEpiSwiGLU).  I must be a multiple of 128.
std::vector<torch::Tensor> gemm_nt_swiglu(torch::Tensor A, torch::Tensor B) {
  check_bf16(A, "A"); check_bf16(B, "B");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_nt_swiglu: shape mismatch");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_nt_swiglu: inner dim must be contiguous");
  const int M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(N % kBN == 0 && K > 0, "gemm_nt_swiglu: [gate; up] rows must be a multiple of 256, K > 0");
  auto gu = torch::empty({M, N}, A.options());
  auto h = torch::empty({M, N / 2}, A.options());
  if (M == 0) return {gu, h};
  c10::cuda::CUDAGuard g(A.device());
  auto ta = make_tmap_2d_bf16(A.data_ptr(), M, K, A.stride(0), 64, GBM);
  auto tb = make_tmap_2d_bf16(B.data_ptr(), N, K, B.stride(0), 64, 128);
  auto a = base_args(M, N, K, gu.data_ptr(), gu.stride(0));
  a.H = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  a.ldh = N / 2;
  // N is a multiple of 256, so both outputs meet the TMA stride rules
  auto tc = make_tmap_2d_bf16(gu.data_ptr(), M, N, gu.stride(0), 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
  auto th = make_tmap_2d_bf16(h.data_ptr(), M, N / 2, N / 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
  a.tma_epi = 1;
  if (use_pair(M, N)) {  // tb already has 128-row boxes (gate / up halves)
    launch_gemm_pair<false, false, kEpiSwiGLU>(ta, tb, tc, &th, a, at::cuda::getCurrentCUDAStream());
    return {gu, h};
  }
  launch_gemm<kBN, kStages, false, false, kEpiSwiGLU>(ta, tb, a, cdiv(M, GBM) * (N / kBN),
                                                      at::cuda::getCurrentCUDAStream(), &tc, &th);
  return {gu, h};
}

// C[M,N] (bf16) = A[M,K] @ B[K,N]
void gemm_nn_out(torch::Tensor A, torch::Tensor B, torch::Tensor C) {
  check_bf16(A, "A"); check_bf16(B, "B"); check_bf16(C, "C");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(0), "gemm_nn: shape mismatch");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm_nn: inner dim must be contiguous");
  const int M = A.size(0), K = A.size(1), N = B.size(1);
  TORCH_CHECK(C.size(0) == M && C.size(1) == N, "gemm_nn: C shape");
  if (M == 0 || N == 0) return;
  if (K == 0) { C.zero_(); return; }
  c10::cuda::CUDAGuard g(A.device());
  auto ta = make_tmap_2d_bf16(A.data_ptr(), M, K, A.stride(0), 64, GBM);
  auto tb = make_tmap_2d_bf16(B.data_ptr(), K, N, B.stride(0), 64, 64);
  auto a = base_args(M, N, K, C.data_ptr(), C.stride(0));
  CUtensorMap tc;
  if (tma_epi_ok(C.data_ptr(), C.stride(0), 2)) {
    tc = make_tmap_2d_bf16(C.data_ptr(), M, N, C.stride(0), 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    a.tma_epi = 1;
  }
  if (a.tma_epi && use_pair(M, N)) {  // tb: 64 x 64 boxes, the same for both kernels
    launch_gemm_pair<false, true, kEpiBF16>(ta, tb, tc, nullptr, a, at::cuda::getCurrentCUDAStream());
    return;
  }
  launch_gemm<kBN, kStages, false, true, kEpiBF16>(ta, tb, a, cdiv(M, GBM) * cdiv(N, kBN),
                                                   at::cuda::getCurrentCUDAStream(),
                                                   a.tma_epi ? &tc : nullptr);
}

torch::Tensor gemm_nn(torch::Tensor A, torch::Tensor B) {
  auto C = torch::empty({A.size(0), B.size(1)}, A.options());
  gemm_nn_out(A, B, C);
  return C;
}

// C[M,N] (fp32) += A[K,M]^T @ B[K,N]
void gemm_tn_acc(torch::Tensor A, torch::Tensor B, torch::Tensor C) {
  check_bf16(A, "A"); check_bf16(B, "B");
  TORCH_CHECK(C.scalar_type() == torch::kFloat32 && C.is_cuda(), "gemm_tn_acc: C must be fp32 CUDA");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(0) == B.size(0), "gemm_tn_acc: shape mismatch");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm_tn_acc: inner dim must be contiguous");
  const int K = A.size(0), M = A.size(1), N = B.size(1);
  TORCH_CHECK(C.size(0) == M && C.size(1) == N, "gemm_tn_acc: C shape");
  if (M == 0 || N == 0 || K == 0) return;
  c10::cuda::CUDAGuard g(A.device());
  auto ta = make_tmap_2d_bf16(A.data_ptr(), K, M, A.stride(0), 64, 64);
  auto tb = make_tmap_2d_bf16(B.data_ptr(), K, N, B.stride(0), 64, 64);
  auto a = base_args(M, N, K, C.data_ptr(), C.stride(0));
  CUtensorMap tc;
  if (tma_epi_ok(C.data_ptr(), C.stride(0), 4)) {
    // C += tile through TMA add-reductions (the read-modify-write happens in L2)
    tc = make_tmap_2d_f32(C.data_ptr(), M, N, C.stride(0), 32, 32);
    a.tma_epi = 1;
  }
  if (a.tma_epi && use_pair(M, N)) {  // ta / tb: 64 x 64 boxes, the same for both kernels
    launch_gemm_pair<true, true, kEpiAccF32>(ta, tb, tc, nullptr, a, at::cuda::getCurrentCUDAStream());
    return;
  }
  launch_gemm<kBN, kStages, true, true, kEpiAccF32>(ta, tb, a, cdiv(M, GBM) * cdiv(N, kBN),
                                                    at::cuda::getCurrentCUDAStream(),
                                                    a.tma_epi ? &tc : nullptr);
}

// ------------------------------------------------------ tensor-parallel GEMMs
// A [M, K] is a full-sequence buffer whose rows [r*tp_rows, (r+1)*tp_rows) are
// written by rank r; B [N, K] (nt) or [K, N] (nn).  The producer waits for
// ag_flags[r] >= ag_seq before loading rows of rank r.
torch::Tensor gemm_ag(torch::Tensor A, torch::Tensor B, bool nn, int64_t ag_flags, int64_t ag_seq,
                      int64_t tp_rows) {
  check_bf16(A, "A"); check_bf16(B, "B");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous(), "gemm_ag: contiguous operands");
  const int M = A.size(0), K = A.size(1);
  const int N = nn ? B.size(1) : B.size(0);
  TORCH_CHECK((nn ? B.size(0) : B.size(1)) == K, "gemm_ag: shape mismatch");
  TORCH_CHECK(tp_rows > 0 && tp_rows % GBM == 0 && M % tp_rows == 0, "gemm_ag: rows per rank must be a multiple of 128");
  auto C = torch::empty({M, N}, A.options());
  if (M == 0 || N == 0) return C;
  c10::cuda::CUDAGuard g(A.device());
  auto ta = make_tmap_2d_bf16(A.data_ptr(), M, K, K, 64, GBM);
  auto a = base_args(M, N, K, C.data_ptr(), N);
  a.ag_flags = reinterpret_cast<const unsigned*>(ag_flags);
  a.ag_seq = static_cast<unsigned>(ag_seq);
  a.tp_rows = static_cast<int>(tp_rows);
  auto st = at::cuda::getCurrentCUDAStream();
  if (nn) {
    auto tb = make_tmap_2d_bf16(B.data_ptr(), K, N, N, 64, 64);
    launch_gemm<kBN, kStages, false, true, kEpiBF16>(ta, tb, a, cdiv(M, GBM) * cdiv(N, kBN), st);
  } else {
    auto tb = make_tmap_2d_bf16(B.data_ptr(), N, K, K, 64, kBN);
    launch_gemm<kBN, kStages, false, false, kEpiBF16>(ta, tb, a, cdiv(M, GBM) * cdiv(N, kBN), st);
  }
  return C;
}

// C = A @ B^T (nt) or A @ B (nn), [M, N] with M the full sequence; row tile of
// owner r goes to rs_dst[r] (that rank's partial plane for this source).
// Returns the grid size (the caller's block counter advances by it).
int64_t gemm_rs(torch::Tensor A, torch::Tensor B, bool nn, std::vector<int64_t> rs_dst, int64_t tp_rows,
                torch::Tensor counter, int64_t counter_before, std::vector<int64_t> flag_dst,
                int64_t flag_idx, int64_t seq) {
  check_bf16(A, "A"); check_bf16(B, "B");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous(), "gemm_rs: contiguous operands");
  const int M = A.size(0), K = A.size(1);
  const int N = nn ? B.size(1) : B.size(0);
  TORCH_CHECK((nn ? B.size(0) : B.size(1)) == K, "gemm_rs: shape mismatch");
  const int world = static_cast<int>(rs_dst.size());
  TORCH_CHECK(world >= 1 && world <= 8 && flag_dst.size() == rs_dst.size(), "gemm_rs: 1..8 ranks");
  TORCH_CHECK(tp_rows > 0 && tp_rows % GBM == 0 && M == tp_rows * world, "gemm_rs: M = tp_rows * world, tp_rows % 128 == 0");
  TORCH_CHECK(N % 32 == 0, "gemm_rs: N must be a multiple of 32");
  c10::cuda::CUDAGuard g(A.device());
  auto ta = make_tmap_2d_bf16(A.data_ptr(), M, K, K, 64, GBM);
  auto a = base_args(M, N, K, nullptr, N);
  a.rs = 1;
  a.tp_world = world;
  a.tp_rows = static_cast<int>(tp_rows);
  for (int r = 0; r < world; ++r) {
    a.rs_dst[r] = reinterpret_cast<__nv_bfloat16*>(rs_dst[r]);
    a.rs_flag_dst[r] = reinterpret_cast<unsigned*>(flag_dst[r]);
    TORCH_CHECK(rs_dst[r] % 16 == 0, "gemm_rs: 16-byte aligned destinations");
  }
  a.rs_flag_idx = static_cast<int>(flag_idx);
  a.rs_seq = static_cast<unsigned>(seq);
  a.rs_counter = reinterpret_cast<unsigned*>(counter.data_ptr());
  const int tiles = cdiv(M, GBM) * cdiv(N, kBN);
  const int grid = std::min(num_sms(), std::max(1, tiles));
  a.rs_target = static_cast<unsigned>(counter_before + grid);
  auto st = at::cuda::getCurrentCUDAStream();
  if (K == 0) TORCH_CHECK(false, "gemm_rs: K must be positive");
  // With NQ_RS_TMA=1 each owner's plane [tp_rows, N] (ld N) becomes a TMA
  // store destination (64-byte row pieces per request instead of 16-byte
  // register stores); the register epilogue is the default.
  RsMaps rsm;
  std::memset(&rsm, 0, sizeof(rsm));
  const RsMaps* rsp = nullptr;
  if (rs_tma_enabled()) {
    for (int r = 0; r < world; ++r)
      rsm.m[r] = make_tmap_2d_bf16(reinterpret_cast<const void*>(rs_dst[r]), tp_rows, N, N, 32, 32,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
    a.tma_epi = 1;
    rsp = &rsm;
  }
  if (nn) {
    auto tb = make_tmap_2d_bf16(B.data_ptr(), K, N, N, 64, 64);
    launch_gemm<kBN, kStages, false, true, kEpiBF16>(ta, tb, a, tiles, st, nullptr, nullptr, rsp);
  } else {
    auto tb = make_tmap_2d_bf16(B.data_ptr(), N, K, K, 64, kBN);
    launch_gemm<kBN, kStages, false, false, kEpiBF16>(ta, tb, a, tiles, st, nullptr, nullptr, rsp);
  }
  return grid;
}

// ------------------------------------------------------------- grouped GEMMs
// X [R, K] rows grouped by `offsets` (multiples of 128), W [G, N, K]:
//   out[r, :] = X[r, :] @ W[g(r)]^T
// Expert-parallel wait arguments of the grouped GEMMs (see GemmArgs): the
// local copy of every source's per-expert counts, this rank's flag slots of
// the exchange channel, the sequence number, the world, E and the first
// local expert.  counts == 0: no wait.
static void set_ep_wait(GemmArgs& a, int64_t counts, int64_t flags, int64_t seq, int64_t world, int64_t E,
                        int64_t expert0) {
  if (counts == 0) return;
  TORCH_CHECK(flags != 0 && world >= 1 && world <= 8 && E > 0, "grouped GEMM: expert-parallel wait arguments");
  a.ep_counts = reinterpret_cast<const int*>(counts);
  a.ep_flags = reinterpret_cast<const unsigned*>(flags);
  a.ep_seq = static_cast<unsigned>(seq);
  a.ep_world = static_cast<int>(world);
  a.ep_E = static_cast<int>(E);
  a.ep_expert0 = static_cast<int>(expert0);
}

torch::Tensor grouped_gemm_nt(torch::Tensor X, torch::Tensor W, torch::Tensor offsets, int64_t ep_counts,
                              int64_t ep_flags, int64_t ep_seq, int64_t ep_world, int64_t ep_E,
                              int64_t ep_expert0) {
  check_bf16(X, "X"); check_bf16(W, "W");
  TORCH_CHECK(W.dim() == 3 && X.size(1) == W.size(2) && W.is_contiguous() && X.is_contiguous(), "grouped_gemm_nt: shapes");
  TORCH_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.numel() == W.size(0) + 1, "offsets");
  const int G = W.size(0), N = W.size(1), K = W.size(2), R = X.size(0);
  TORCH_CHECK(G <= kMaxGroups, "too many groups");
  auto C = torch::empty({R, N}, X.options());
  if (R == 0) return C;
  c10::cuda::CUDAGuard gd(X.device());
  auto ta = make_tmap_2d_bf16(X.data_ptr(), R, K, K, 64, GBM);
  auto tb = make_tmap_2d_bf16(W.data_ptr(), static_cast<int64_t>(G) * N, K, K, 64, kBN);
  auto a = base_args(R, N, K, C.data_ptr(), N);
  a.group_mode = kGroupM; a.num_groups = G; a.offsets = offsets.data_ptr<int>(); a.b_group_rows = N;
  set_ep_wait(a, ep_counts, ep_flags, ep_seq, ep_world, ep_E, ep_expert0);
  launch_gemm<kBN, kStages, false, false, kEpiBF16>(ta, tb, a, cdiv(R, GBM) * cdiv(N, kBN),
                                                    at::cuda::getCurrentCUDAStream());
  return C;
}

// dY [R, N] grouped rows, W [G, N, K]: out[r, :] = dY[r, :] @ W[g(r)]   ([R, K])
torch::Tensor grouped_gemm_nn(torch::Tensor dY, torch::Tensor W, torch::Tensor offsets, int64_t ep_counts,
                              int64_t ep_flags, int64_t ep_seq, int64_t ep_world, int64_t ep_E,
                              int64_t ep_expert0) {
  check_bf16(dY, "dY"); check_bf16(W, "W");
  TORCH_CHECK(W.dim() == 3 && dY.size(1) == W.size(1) && W.is_contiguous() && dY.is_contiguous(), "grouped_gemm_nn: shapes");
  const int G = W.size(0), N = W.size(1), K = W.size(2), R = dY.size(0);
  TORCH_CHECK(N % 64 == 0, "grouped_gemm_nn: per-group reduction extent must be a multiple of 64");
  auto C = torch::empty({R, K}, dY.options());
  if (R == 0) return C;
  c10::cuda::CUDAGuard gd(dY.device());
  auto ta = make_tmap_2d_bf16(dY.data_ptr(), R, N, N, 64, GBM);
  auto tb = make_tmap_2d_bf16(W.data_ptr(), static_cast<int64_t>(G) * N, K, K, 64, 64);
  auto a = base_args(R, K, N, C.data_ptr(), K);
  a.group_mode = kGroupM; a.num_groups = G; a.offsets = offsets.data_ptr<int>(); a.b_group_rows = N;
  set_ep_wait(a, ep_counts, ep_flags, ep_seq, ep_world, ep_E, ep_expert0);
  launch_gemm<kBN, kStages, false, true, kEpiBF16>(ta, tb, a, cdiv(R, GBM) * cdiv(K, kBN),
                                                   at::cuda::getCurrentCUDAStream());
  return C;
}

// dW[g] (fp32 [N, K]) += dY[rows of g]^T @ X[rows of g]
void grouped_gemm_tn_acc(torch::Tensor dY, torch::Tensor X, torch::Tensor dW, torch::Tensor offsets) {
  check_bf16(dY, "dY"); check_bf16(X, "X");
  TORCH_CHECK(dW.scalar_type() == torch::kFloat32 && dW.dim() == 3 && dW.is_contiguous(), "dW");
  const int G = dW.size(0), N = dW.size(1), K = dW.size(2), R = dY.size(0);
  TORCH_CHECK(dY.size(1) == N && X.size(1) == K && X.size(0) == R, "grouped_gemm_tn_acc: shapes");
  if (R == 0) return;
  c10::cuda::CUDAGuard gd(dY.device());
  auto ta = make_tmap_2d_bf16(dY.data_ptr(), R, N, N, 64, 64);
  auto tb = make_tmap_2d_bf16(X.data_ptr(), R, K, K, 64, 64);
  auto a = base_args(N, K, 0, dW.data_ptr(), K);
  a.group_mode = kGroupK; a.num_groups = G; a.offsets = offsets.data_ptr<int>();
  a.c_group_stride = static_cast<int64_t>(N) * K;
  launch_gemm<kBN, kStages, true, true, kEpiAccF32>(ta, tb, a, G * cdiv(N, GBM) * cdiv(K, kBN),
                                                    at::cuda::getCurrentCUDAStream());
}

}  // namespace nq
