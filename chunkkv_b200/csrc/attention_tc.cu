// Attention of the recomputed tokens over the blended cache on tcgen05/TMEM
// (torch_engine.py:68-70 with the mask of torch_engine.py:157).
//
// Query row (token t, head g) sees key j iff j <= positions[t].  GQA: the G =
// Hq/Hk heads sharing a KV head are packed as consecutive rows; a Q tile holds
// T = floor(128/G) tokens x G heads (126 rows at G = 7) and a CTA holds two Q
// tiles of one KV head, so every K/V tile it loads serves 2T tokens x G heads.
// Per key tile j (128 keys) and Q tile w in {0, 1}:
//   S_w = Q_w K_j^T   tcgen05.mma (A = Q_w, B = K tile, both K-major in smem), fp32
//                     into TMEM columns [128w, 128w+128)
//   softmax           warpgroup w, one thread per row (= TMEM lane): the S row in one
//                     128-column TMEM load, position mask, online max/sum in fp32 with
//                     ex2 (scale folded in); O_w is rescaled in TMEM only when the
//                     running max grows by more than 2^8 (lazy: O and l always share
//                     the same max, so the result is exact)
//   P_w (bf16)        stored back over S_w in TMEM (two values per column)
//   O_w += P_w V_j    tcgen05.mma with A read from TMEM, B = V tile read MN-major (the
//                     cache stores V as [key][d], d contiguous), fp32 in TMEM
// The two Q tiles interleave on the tensor core: while warpgroup 0 runs the softmax of
// tile j the tensor core runs P_1 V_{j-1} and S_1(j), and the other way round.  The
// warpgroups are not made to take turns: once the MMA issue is its own warp, two
// softmax warpgroups running side by side hide each other's latencies (measured
// 5-8 % faster than strict alternation).  tcgen05.mma ops of one thread execute in
// issue order, so S_w(j+1) may be issued right after P_w(j) V_j, which reads the same
// TMEM columns.  K and V stages are released
// separately (K after both S, V after both P.V).
// Warps: 0..3 and 4..7 = softmax / correction / epilogue of Q tiles 0 and 1,
// 8 = TMA producer, 9 = MMA issuer + TMEM owner.  A softmax thread reads its S row
// from TMEM twice, 64 columns at a time (row max, then exponentials), so it never
// holds more than half a row.  The exponentials run on the MUFU unit (ex2.approx, 16
// results per clock per SM); moving a share of them to a polynomial on the FMA pipe
// was slower once the two warpgroups overlap (issue-bound, not MUFU-bound).  Every
// wait is bounded (ckv_common.cuh).
// The kernel is persistent: one CTA per SM runs work items (row block, KV head, key
// split) one after another on the same TMEM allocation and barriers.  The producer warp
// claims items from a counter in the workspace and publishes them, with their tokens'
// positions, through a small ring in shared memory.  It loads each Q tile by TMA (a 3-D
// box of G heads x T tokens lands as the packed rows) as soon as the current item's
// last S MMA on that tile is done, so the next item's first S MMA overlaps this item's
// last P V and its epilogue.  Each Q tile has its own "O complete" barrier, so one
// warpgroup's epilogue never waits for the other's last tile.
#include <algorithm>
#include <mutex>
#include <vector>

#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(attention_tc)

namespace ckv {
namespace {

constexpr int BM = 128;  // rows per Q tile (packed token x head)
constexpr int NQ = 2;    // Q tiles per CTA
constexpr int BN = 128;  // keys per tile
constexpr int KS = 2;    // K stages
constexpr int VS = 2;    // V stages
constexpr int kThreads = NQ * 128 + 64;  // two softmax warpgroups + producer + MMA warps
constexpr int kWarpTma = 8, kWarpMma = 9;
constexpr uint32_t TMEM_COLS = 512;  // S/P of tile w at [128w, 128w+128), O of tile w at 256+128w
constexpr uint32_t O_COL = 256;
constexpr uint32_t ATOM_BYTES = 128 * 128;  // one [128 rows][64 bf16] swizzle-128 atom
constexpr float kRescaleThreshold = 8.0f;   // log2 units

template <int HD>
struct Cfg {
  static constexpr int ATOMS = HD / 64;
  static constexpr uint32_t Q_BYTES = BM * HD * 2;
  // bytes one Q tile's TMA boxes deliver: G heads x T tokens x HD (rows past G * T stay)
  __host__ __device__ static constexpr uint32_t Q_TX(int g, int t) { return uint32_t(HD) * g * t * 2; }
  static constexpr uint32_t KV_TILE = BN * HD * 2;
  // at least 120 KiB so two CTAs never share an SM: each allocates all 512 TMEM columns
  // + item ring (4 x 32 B) with its token positions (4 x NQ x BM ints), the softmax
  // warps' store staging tiles (8 x 32 rows x 80 B), barriers and flags
  static constexpr uint32_t SMEM_NEED = 1024 + NQ * Q_BYTES + (KS + VS) * KV_TILE + 4096 + 20480 + 512;
  static constexpr uint32_t SMEM = SMEM_NEED > 120 * 1024 ? SMEM_NEED : 120 * 1024;
  static constexpr uint32_t IDESC_S = umma_idesc_bf16(BM, BN);
  static constexpr uint32_t IDESC_PV = umma_idesc_bf16(BM, HD) | (1u << 16);  // B MN-major
};

// all lanes wait; the warp agrees on the outcome so collective TMEM ops stay converged
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort, &g_err_word);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitLimitNs) break;
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Work items: (row block rb, KV head hk, key split z).  Slots come in groups of one
// per (head, row block), row blocks from the last (longest) one down; group gi holds
// split z = n_split - max_splits + gi of the block, so a block's last split, the only
// one shorter than tps key tiles, is in the last group, and the longest blocks' full
// splits come first: roughly longest first over the whole grid.  A slot with z < 0 (a
// block with fewer splits) is empty and skipped.
struct Item {
  int rb, hk, split, n_split, kt0, n_kt, pad0, pad1;  // rb < 0: no more work
};
constexpr int kItemSlots = 4;  // ring of items published by the producer warp
// Epilogue staging: per softmax warp 32 rows x 16 words, rows padded to 20 words (80 B)
// so that the 16-byte writes of eight consecutive lanes fall in distinct banks
constexpr int kStageStride = 20;
constexpr uint32_t kStageBytes = NQ * 4 * 32 * kStageStride * 4;
static_assert(kItemSlots * (sizeof(Item) + NQ * BM * sizeof(int)) + kStageBytes + 40 * sizeof(uint64_t) + 8 <=
                  4096 + 20480 + 512,
              "item ring, positions, staging and barriers must fit the shared-memory reserve");

// 10 warps: two of the four SM sub-partitions hold three warps, so the register
// file allows at most 16384 / (3 * 32) = 170 registers per thread.
// Persistent: one CTA per SM keeps its TMEM, barriers and pipeline across items.  With
// `sched` (two zeroed words: next slot, CTAs done) CTAs take slots from an atomic
// counter, and the last CTA to run out of work sets both words back to 0; without it
// CTA c takes slots c, c + gridDim.x, ...
template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmQ, const int32_t* __restrict__ positions,
                        uint16_t* __restrict__ out, int M, int Hq, int Hk, int n_ctx, float scale_log2,
                        int tps, int max_splits, int blocks, unsigned* __restrict__ sched,
                        float* __restrict__ part_o, float2* __restrict__ part_ml) {
  using C = Cfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                      // [NQ][Q_BYTES]
  uint8_t* sK = sQ + NQ * C::Q_BYTES;      // [KS][KV_TILE]
  uint8_t* sV = sK + KS * C::KV_TILE;      // [VS][KV_TILE]
  Item* items = reinterpret_cast<Item*>(sV + VS * C::KV_TILE);  // [kItemSlots]
  int* s_pos = reinterpret_cast<int*>(items + kItemSlots);      // [kItemSlots][NQ * BM] token positions
  uint32_t* s_stage = reinterpret_cast<uint32_t*>(s_pos + kItemSlots * NQ * BM);  // [8 warps][32][20]
  uint64_t* k_full = reinterpret_cast<uint64_t*>(s_stage + kStageBytes / 4);
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;  // [NQ]
  uint64_t* p_full = s_full + NQ;   // [NQ]
  uint64_t* o_done = p_full + NQ;   // [NQ]
  uint64_t* q_ready = o_done + NQ;  // [NQ]: Q tile w of the next item landed (TMA)
  uint64_t* q_free = q_ready + NQ;  // [NQ]: the current item's last S MMA of tile w is done
  uint64_t* o_full = q_free + NQ;   // [NQ]: the current item's last P V of tile w is done
  uint64_t* item_full = o_full + NQ;  // [kItemSlots]
  uint64_t* item_empty = item_full + kItemSlots;  // [kItemSlots]
  uint64_t* drain = item_empty + kItemSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = Hq / Hk;
  const int T = BM / G;  // tokens per Q tile
  const int n_slots = blocks * Hk * max_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int w = 0; w < NQ; ++w) {
      mbar_init(&s_full[w], 1);
      mbar_init(&p_full[w], 128);
      mbar_init(&o_done[w], 1);
      mbar_init(&q_ready[w], 1);
      mbar_init(&q_free[w], 1);
      mbar_init(&o_full[w], 1);
    }
    for (int s = 0; s < kItemSlots; ++s) {
      mbar_init(&item_full[s], 1);
      mbar_init(&item_empty[s], 1 + NQ * 4);  // the MMA thread and each softmax warp
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
    fence_async_smem();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmQ);
  }
  // Q rows past G * T (padding of a tile) are never loaded: zero them once
  for (int i = threadIdx.x; i < NQ * C::ATOMS * (BM - G * T) * 8; i += kThreads) {
    const int per_atom = (BM - G * T) * 8;  // 16-byte chunks
    const int wa = i / per_atom, c = i - wa * per_atom;
    *reinterpret_cast<uint4*>(sQ + wa * ATOM_BYTES + (G * T) * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  fence_async_smem();
  if (warp == kWarpMma) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // set-up done; q, the caches, the positions and the workspace belong to the kernels
  // before (dependent launch)
  pdl_wait();
  pdl_launch_next();

  if (warp == kWarpTma) {
    // ------------------------------------------- item scheduler + TMA producer (one warp)
    int it = 0;          // items published
    int nk = 0, nv = 0;  // K / V tile loads issued (all items)
    int nq[NQ] = {};     // Q tile loads issued per tile
    int cursor = blockIdx.x;
    bool ok = true;
    while (ok) {
      // next non-empty slot: the warp reads the block's positions for its last key tile
      Item rec{-1, 0, 0, 0, 0, 0, 0, 0};
      int pv[NQ * BM / 32];  // the item's token positions, lane + 32 j (clamped)
      while (true) {
        int slot = cursor;
        if (sched != nullptr) {
          if (lane == 0) slot = int(atomicAdd(&sched[0], 1u));
          slot = __shfl_sync(0xffffffffu, slot, 0);
        } else {
          cursor += gridDim.x;
        }
        if (slot >= n_slots) break;
        const int gi = slot / (Hk * blocks);  // slot group
        const int rem = slot - gi * (Hk * blocks);
        const int hk = rem / blocks;
        const int rb = blocks - 1 - (rem - hk * blocks);
        const int t0 = rb * NQ * T;
        const int n_tok = min(NQ * T, M - t0);
        int mx = 0;
#pragma unroll
        for (int j = 0; j < NQ * BM / 32; ++j) {
          const int i = lane + 32 * j;
          int p = 0;
          if (i < n_tok) {
            p = positions[t0 + i];
            if (p < 0 || p >= n_ctx) {
              if (gi == 0 && hk == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
              p = p < 0 ? 0 : n_ctx - 1;
            }
          }
          pv[j] = p;
          mx = max(mx, p);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const int kt_all = mx / BN + 1;  // key tiles 0 .. last visible key
        const int n_split = (kt_all + tps - 1) / tps;
        // group gi holds split n_split - max_splits + gi of every block that has one: the
        // full-size splits of the longest blocks go out first and every block's last
        // (shortest) split in the last group, so the work left at the end is small
        const int z = n_split - max_splits + gi;
        if (z >= 0) {
          rec = Item{rb, hk, z, n_split, z * tps, min(tps, kt_all - z * tps), 0, 0};
          break;
        }
      }
      // publish the record and its positions (a record with rb < 0 tells the consumers
      // to stop), then load its Q tiles and its K/V tiles
      const int s = it % kItemSlots;
      bool free_slot = true;
      if (lane == 0) free_slot = mbar_wait(&item_empty[s], ((it / kItemSlots) & 1) ^ 1, abort, &g_err_word);
      if (!__shfl_sync(0xffffffffu, free_slot ? 1 : 0, 0)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int j = 0; j < NQ * BM / 32; ++j) s_pos[s * NQ * BM + lane + 32 * j] = pv[j];
      __threadfence_block();
      __syncwarp();
      if (lane == 0) {
        items[s] = rec;
        mbar_arrive(&item_full[s]);
        // Q tile w of this item, once the previous item's last S MMA on tile w is done
        for (int w = 0; w < NQ && ok && rec.rb >= 0; ++w) {
          if (it > 0 && !mbar_wait(&q_free[w], (it - 1) & 1, abort, &g_err_word)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&q_ready[w], C::Q_TX(G, T));
          ++nq[w];
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a)
            tma_load_3d(sQ + w * C::Q_BYTES + a * ATOM_BYTES, &tmQ, a * 64, rec.hk * G,
                        rec.rb * NQ * T + w * T, &q_ready[w]);
        }
        for (int j = 0; j < rec.n_kt && ok && rec.rb >= 0; ++j) {
          const int gk = nk;
          if (!mbar_wait(&k_empty[gk % KS], ((gk / KS) & 1) ^ 1, abort, &g_err_word)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&k_full[gk % KS], C::KV_TILE);
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a)
            tma_load_3d(sK + (gk % KS) * C::KV_TILE + a * ATOM_BYTES, &tmK, a * 64, (rec.kt0 + j) * BN, rec.hk,
                        &k_full[gk % KS]);
          ++nk;
          const int gv = nv;
          if (!mbar_wait(&v_empty[gv % VS], ((gv / VS) & 1) ^ 1, abort, &g_err_word)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&v_full[gv % VS], C::KV_TILE);
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a)
            tma_load_3d(sV + (gv % VS) * C::KV_TILE + a * ATOM_BYTES, &tmV, a * 64, (rec.kt0 + j) * BN, rec.hk,
                        &v_full[gv % VS]);
          ++nv;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (rec.rb < 0) break;
      ++it;
    }
    if (lane == 0) {
      if (!ok) {  // aborted: let the copies already issued land
        for (int i = (nk > KS ? nk - KS : 0); i < nk; ++i) drain_wait(&k_full[i % KS], (i / KS) & 1);
        for (int i = (nv > VS ? nv - VS : 0); i < nv; ++i) drain_wait(&v_full[i % VS], (i / VS) & 1);
        for (int w = 0; w < NQ; ++w)
          if (nq[w] > 0) drain_wait(&q_ready[w], (nq[w] - 1) & 1);
      }
      if (sched != nullptr) {
        // every CTA arrives here once, after its last claim on the slot counter; the
        // last one leaves both words at 0 for the next launch
        if (atomicAdd(&sched[1], 1u) == gridDim.x - 1) {
          atomicExch(&sched[0], 0u);
          atomicExch(&sched[1], 0u);
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      auto issue_s = [&](int w, int gt, bool last) {
        const uint32_t q0 = smem_u32(sQ + w * C::Q_BYTES);
        const uint32_t k0 = smem_u32(sK + (gt % KS) * C::KV_TILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
          tc_mma_f16(tmem + w * BN, umma_desc_sw128(q0 + off), umma_desc_sw128(k0 + off), C::IDESC_S,
                     kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[w]);
        if (last) tc_commit(&q_free[w]);  // Q tile w may be overwritten for the next item
      };
      auto issue_pv = [&](int w, int gt, bool first) {
        const uint32_t v0 = smem_u32(sV + (gt % VS) * C::KV_TILE);
        const uint32_t pbuf = tmem + w * BN;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          tc_mma_f16_ts(tmem + O_COL + w * 128, pbuf + kk * 8, umma_desc_sw128_mn(v0 + kk * 16 * 128, ATOM_BYTES),
                        C::IDESC_PV, (!first || kk > 0) ? 1u : 0u);
        tc_commit(&o_done[w]);
      };
      bool ok = true;
      int g = 0;  // key tiles consumed (all items)
      for (int it = 0; ok; ++it) {
        const int s = it % kItemSlots;
        if (!mbar_wait(&item_full[s], (it / kItemSlots) & 1, abort, &g_err_word)) {
          ok = false;
          break;
        }
        const int n_kt = items[s].rb < 0 ? -1 : items[s].n_kt;
        mbar_arrive(&item_empty[s]);
        if (n_kt < 0) break;
        // S of the first tile, per Q tile as soon as that tile's Q is in smem
        if (!mbar_wait(&k_full[g % KS], (g / KS) & 1, abort, &g_err_word)) {
          ok = false;
          break;
        }
        for (int w = 0; w < NQ && ok; ++w) {
          if (!mbar_wait(&q_ready[w], it & 1, abort, &g_err_word)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(w, g, n_kt == 1);
        }
        if (!ok) break;
        tc_commit(&k_empty[g % KS]);
        for (int j = 0; j < n_kt && ok; ++j) {
          const int gt = g + j, nxt = gt + 1;
          for (int w = 0; w < NQ && ok; ++w) {
            if (!mbar_wait(&p_full[w], gt & 1, abort, &g_err_word) ||
                (w == 0 && !mbar_wait(&v_full[gt % VS], (gt / VS) & 1, abort, &g_err_word))) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(w, gt, j == 0);
            if (j + 1 == n_kt) tc_commit(&o_full[w]);  // O of tile w is final
            if (w == NQ - 1) tc_commit(&v_empty[gt % VS]);
            if (j + 1 < n_kt) {
              if (w == 0 && !mbar_wait(&k_full[nxt % KS], (nxt / KS) & 1, abort, &g_err_word)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_s(w, nxt, j + 2 == n_kt);
              if (w == NQ - 1) tc_commit(&k_empty[nxt % KS]);
            }
          }
        }
        g += n_kt;
      }
      if (!ok) {
        tc_commit(drain);
        drain_wait(drain, 0);
      }
    }
  } else {
    // ------------------------------------------------- softmax / correction / epilogue
    const int w = warp >> 2;         // Q tile of this warpgroup
    const int sub = warp & 3;        // TMEM sub-partition (lanes 32*sub .. +31)
    const int r = sub * 32 + lane;   // row in the Q tile == TMEM lane
    const int tr = r / G;           // token of the row in the Q tile
    const uint32_t lane_base = tmem + (uint32_t(sub * 32) << 16);
    const uint32_t sbuf = lane_base + w * BN;
    const uint32_t obuf = lane_base + O_COL + w * 128;

    // this thread's row of an item: token, its position, whether the row is real
    struct Row {
      int tok, pos;
      bool valid;
    };
    // item `it` from the ring with this thread's row of it (the position comes from the
    // ring's copy, read before the slot is released); one lane per warp releases it
    auto take = [&](int it, Item& rec, Row& x) -> bool {
      const int s = it % kItemSlots;
      if (!warp_wait(&item_full[s], (it / kItemSlots) & 1, abort)) return false;
      rec = items[s];
      const int n_tok = min(NQ * T, M - rec.rb * NQ * T);
      const int tt = w * T + tr;  // token index in the item
      x.valid = rec.rb >= 0 && r < T * G && tt < n_tok;
      x.tok = rec.rb * NQ * T + (x.valid ? tt : 0);
      // padding rows see every key: they never force the masked path on their warp
      x.pos = x.valid ? s_pos[s * NQ * BM + tt] : n_ctx - 1;
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[s]);
      return true;
    };

    Item cur;
    Row row{0, 0, false};
    bool ok = take(0, cur, row);
    int g = 0;  // key tiles consumed (all items)
    for (int it = 0; ok && cur.rb >= 0; ++it) {
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < cur.n_kt; ++j) {
        const int gt = g + j;
        if (!warp_wait(&s_full[w], gt & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int lim = row.pos - (cur.kt0 + j) * BN;  // keys at index > lim are masked
        const bool full = __all_sync(0xffffffffu, lim >= BN - 1);  // whole tile visible to the warp
        // pass 1: row max of the raw scores (scale > 0 commutes with max), 64 columns at a
        // time, 8 chains of 3-input max
        float mx8[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) mx8[c] = -INFINITY;
#pragma unroll
        for (int h = 0; h < BN / 64; ++h) {
          uint32_t u[64];
          tmem_ld64w(sbuf + 64 * h, u);
          if (!full) {
#pragma unroll
            for (int e = 0; e < 64; ++e)
              if (64 * h + e > lim) u[e] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int c = 0; c < 8; ++c)
              mx8[c] = max3f(mx8[c], __uint_as_float(u[16 * k + 2 * c]), __uint_as_float(u[16 * k + 2 * c + 1]));
        }
        const float mx = fmaxf(max3f(mx8[0], mx8[1], mx8[2]), max3f(max3f(mx8[3], mx8[4], mx8[5]), mx8[6], mx8[7]));
        const float m_new = fmaxf(m, mx * scale_log2);
        const bool need = j > 0 && m_new > m + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          // O may be touched only after P(j-1) V(j-1) has landed
          if (!warp_wait(&o_done[w], (gt - 1) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float corr = need ? ex2_approx(m - m_new) : 1.0f;
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            float o[32];
            tmem_ld32(obuf + c, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= corr;
            tmem_st32(obuf + c, o);
          }
          l *= corr;
        }
        if (j == 0 || need) m = m_new;
        // pass 2: P = 2^(s*scale - m) (scale folded into one packed FFMA), 64 columns at a
        // time, written back over S as bf16 pairs: P of keys 64h.. goes to columns 32h..,
        // whose scores were read in the half before.  Masked scores are -inf and give
        // exactly 0.  A row that has seen no visible key yet (possible in a later key
        // split) keeps m = -inf; the finite base keeps its P at exactly 0 instead of NaN.
        const float neg_m = m == -INFINITY ? 0.f : -m;
        const float2 sc2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(neg_m, neg_m);
        float2 rs4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) rs4[i] = make_float2(0.f, 0.f);
#pragma unroll
        for (int h = 0; h < BN / 64; ++h) {
          uint32_t u[64];
          tmem_ld64w(sbuf + 64 * h, u);
          if (full) {
#pragma unroll
            for (int pr = 0; pr < 32; ++pr) {
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(u[2 * pr]), __uint_as_float(u[2 * pr + 1])), sc2, nm2);
              const float2 pv = make_float2(ex2_approx(x.x), ex2_approx(x.y));
              rs4[pr & 3] = __fadd2_rn(rs4[pr & 3], pv);
              u[pr] = pack_bf2(pv.x, pv.y);
            }
          } else {
#pragma unroll
            for (int pr = 0; pr < 32; ++pr) {
              const float s0 = 64 * h + 2 * pr <= lim ? __uint_as_float(u[2 * pr]) : -INFINITY;
              const float s1 = 64 * h + 2 * pr + 1 <= lim ? __uint_as_float(u[2 * pr + 1]) : -INFINITY;
              const float2 x = __ffma2_rn(make_float2(s0, s1), sc2, nm2);
              const float2 pv = make_float2(ex2_approx(x.x), ex2_approx(x.y));
              rs4[pr & 3] = __fadd2_rn(rs4[pr & 3], pv);
              u[pr] = pack_bf2(pv.x, pv.y);
            }
          }
          tmem_st32u(sbuf + 32 * h, *reinterpret_cast<const uint32_t(*)[32]>(u));
        }
        const float2 rsum = __fadd2_rn(__fadd2_rn(rs4[0], rs4[1]), __fadd2_rn(rs4[2], rs4[3]));
        l += rsum.x + rsum.y;
        tc_fence_before();
        mbar_arrive(&p_full[w]);
      }
      if (!ok) break;
      g += cur.n_kt;
      // the next item's record (its Q tiles are already on their way by TMA), then
      // this item's epilogue once its last P V on this tile is done
      Item nxt;
      Row nrow{0, 0, false};
      ok = take(it + 1, nxt, nrow);
      if (!ok || !warp_wait(&o_full[w], it & 1, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t* stg = s_stage + warp * (32 * kStageStride);
      if (cur.n_split > 1) {
        // One slice of the keys: unnormalised O with its (max, sum), merged by the combine
        // kernel.  The partials of a warpgroup are stored column-chunk-major (8 fp32
        // columns of all 128 rows per chunk, the two 16-byte halves of row r swapped when
        // bit 2 of r is set), so the warp's 32 rows of one chunk are 1 KiB of contiguous
        // global memory.  Each chunk is staged in one of the warp's two 1 KiB buffers and
        // written by a TMA bulk store; the staging of the next chunk overlaps it.  Plain
        // per-lane stores of the same partials took about four times as long here.
        const int64_t blk = (int64_t((cur.rb * Hk + cur.hk) * max_splits + cur.split) * NQ + w) * BM * HD;
        float* gdst = part_o + blk + sub * 32 * 8;
        uint8_t* stg8 = reinterpret_cast<uint8_t*>(stg);
        const int swz = (lane >> 2) & 1;
        int chunk = 0;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          float o[32];
          tmem_ld32(obuf + c, o);
#pragma unroll
          for (int h = 0; h < 4; ++h, ++chunk) {
            uint8_t* buf = stg8 + (chunk & 1) * 1024;
            if (chunk >= 2) {  // the store that last read this buffer has read it
              if (lane == 0) bulk_wait_read<1>();
              __syncwarp();
            }
            float4* mine = reinterpret_cast<float4*>(buf + lane * 32);
            mine[swz] = make_float4(o[8 * h], o[8 * h + 1], o[8 * h + 2], o[8 * h + 3]);
            mine[swz ^ 1] = make_float4(o[8 * h + 4], o[8 * h + 5], o[8 * h + 6], o[8 * h + 7]);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              bulk_store(gdst + (c / 8 + h) * (BM * 8), buf, 1024);
              bulk_commit();
            }
          }
        }
        if (lane == 0) bulk_wait_read<0>();  // both buffers free for the next epilogue
        __syncwarp();
        if (row.valid) {
          const int64_t prow = int64_t((cur.rb * Hk + cur.hk) * max_splits + cur.split) * (NQ * BM) + w * BM + r;
          part_ml[prow] = make_float2(m, l);
        }
      } else {
        // Stores go through this warp's staging tile: a lane holds one row (TMEM lane) of
        // O, and a store whose 32 lanes hit 32 rows is replayed once per row.  So 16 words
        // of each row (32 bf16 outputs) are staged, then written four lanes per row, eight
        // rows per instruction.  dst[k]: element offset in out of the first column of this
        // warp's row 8k + lane / 4, -1 for padding rows and rows past M.
        int64_t dst[4];
        {
          const int t0 = cur.rb * NQ * T;
          const int n_tok = min(NQ * T, M - t0);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int rq = sub * 32 + 8 * k + (lane >> 2);
            const int tq = rq / G, gq = rq - tq * G, ttq = w * T + tq;
            const bool vq = rq < T * G && ttq < n_tok;
            dst[k] = !vq ? -1 : (int64_t(t0 + ttq) * Hq + cur.hk * G + gq) * HD;
          }
        }
        auto flush = [&](const uint32_t(&v)[16], int col) {
          uint4* mine = reinterpret_cast<uint4*>(stg + lane * kStageStride);
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) mine[qd] = make_uint4(v[4 * qd], v[4 * qd + 1], v[4 * qd + 2], v[4 * qd + 3]);
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint4 x = reinterpret_cast<const uint4*>(stg + (8 * k + (lane >> 2)) * kStageStride)[lane & 3];
            if (dst[k] >= 0) *reinterpret_cast<uint4*>(out + dst[k] + col + (lane & 3) * 8) = x;
          }
          __syncwarp();
        };
        const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          float o[32];
          tmem_ld32(obuf + c, o);
          uint32_t v[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = pack_bf2(o[2 * e] * inv, o[2 * e + 1] * inv);
          flush(v, c);
        }
      }
      // O has been read: the next item's first P V (which overwrites it) is issued only
      // after this warpgroup's next p_full
      tc_fence_before();
      cur = nxt;
      row = nrow;
    }
    // the split partials' bulk stores have written global memory before the CTA ends
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Merge the key splits of the row blocks that were split: O = sum_s 2^(m_s - M) O_s /
// sum_s 2^(m_s - M) l_s with M = max_s m_s (all in the log2 domain of the kernel).
// A warp takes kCombineRows packed rows; for each, lane s reads split s's (m, l), then
// each lane sums its four columns over the splits, the loads of all its rows in flight
// together (one wave of CTAs at the 7B shape).  Rows of unsplit blocks were written
// directly.
constexpr int kCombineWarps = 8;
constexpr int kCombineRows = 4;
template <int HD>
__global__ void __launch_bounds__(kCombineWarps * 32, 4) attention_combine_kernel(
    const int32_t* __restrict__ positions, uint16_t* __restrict__ out, int M, int Hq, int Hk, int n_ctx,
    int tps, int max_splits, const float* __restrict__ part_o, const float2* __restrict__ part_ml) {
  pdl_wait();  // the partials come from the attention kernel just before (dependent launch)
  pdl_launch_next();
  constexpr int R = kCombineRows;
  const int G = Hq / Hk;
  const int T = BM / G;
  constexpr int kChunks = NQ * BM / (kCombineWarps * R);  // CTAs per (row block, KV head)
  const int rb = blockIdx.x / kChunks, chunk = blockIdx.x - rb * kChunks, hk = blockIdx.y;
  const int t0 = rb * NQ * T;
  const int n_tok = min(NQ * T, M - t0);
  __shared__ int s_max;
  if (threadIdx.x == 0) s_max = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n_tok; i += blockDim.x)
    atomicMax(&s_max, min(max(positions[t0 + i], 0), n_ctx - 1));
  __syncthreads();
  const int n_split = ((s_max + BN) / BN + tps - 1) / tps;
  if (n_split <= 1) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t stride = NQ * BM;
  const int64_t blk = int64_t((rb * Hk + hk) * max_splits);
  // lane v < HD / 4 takes columns 4v .. 4v + 3: 16-byte half (v & 1) of 8-column chunk
  // v >> 1, stored swapped with the other half when bit 2 of the row is set (the
  // kernel's column-chunk-major partial layout)
  const bool mine = lane < HD / 4;
  float wgt[R], inv[R];
  int off[R];
  int64_t orow[R];
  bool ok[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int pr = (chunk * kCombineWarps + warp) * R + i;
    const int w = pr / BM, r = pr - w * BM;
    const int tr = r / G, g = r - tr * G, tt = w * T + tr;
    ok[i] = r < T * G && tt < n_tok;  // the same for the whole warp
    const float2 ml =
        ok[i] && lane < n_split ? part_ml[blk * stride + pr + lane * stride] : make_float2(-INFINITY, 0.f);
    float mmax = ml.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, o));
    wgt[i] = ok[i] && lane < n_split ? exp2f(ml.x - mmax) : 0.f;
    float L = wgt[i] * ml.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    inv[i] = L > 0.f ? 1.0f / L : 0.f;
    off[i] = w * (BM * HD) + (lane >> 1) * (BM * 8) + r * 8 + (((lane & 1) ^ ((r >> 2) & 1)) << 2);
    orow[i] = (int64_t(t0 + tt) * Hq + hk * G + g) * HD;
  }
  const float* po = part_o + blk * NQ * BM * HD;
  float4 acc[R];
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 2
  for (int sp = 0; sp < n_split; ++sp) {
    const float* ps = po + int64_t(sp) * NQ * BM * HD;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const float ws = __shfl_sync(0xffffffffu, wgt[i], sp);
      if (mine && ok[i]) {
        const float4 x = *reinterpret_cast<const float4*>(ps + off[i]);
        acc[i].x = fmaf(ws, x.x, acc[i].x);
        acc[i].y = fmaf(ws, x.y, acc[i].y);
        acc[i].z = fmaf(ws, x.z, acc[i].z);
        acc[i].w = fmaf(ws, x.w, acc[i].w);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < R; ++i)
    if (mine && ok[i])
      *reinterpret_cast<uint2*>(out + orow[i] + 4 * lane) =
          make_uint2(pack_bf2(acc[i].x * inv[i], acc[i].y * inv[i]), pack_bf2(acc[i].z * inv[i], acc[i].w * inv[i]));
}

// Key-split plan: split only when the unsplit grid leaves SMs idle.
struct SplitPlan {
  int tps, max_splits, blocks;
  int64_t bytes;  // partial O and (max, sum) of every split item
};
// The workspace starts with the scheduler's two words (next slot, CTAs done), padded to
// 256 bytes; the split partials follow.
constexpr int64_t kSchedBytes = 256;
// Fixed cost of one item, in key-tile times, for the persistent kernel: its first S
// MMA and the epilogue are only partly hidden behind the neighbouring items; a split
// item also writes its fp32 partial O.
constexpr double kItemCost = 0.7;
constexpr double kSplitItemCost = 1.0;
// Estimated makespan, in key-tile times, of a split plan: the list-scheduling estimate
// total work / SMs + half the largest item (items go out roughly largest first), plus,
// when split, the combine (reading every partial at the HBM rate: one tile time per
// 14.3 MB).  Row block b is assumed to reach position (b + 1) / blocks * n_ctx (sorted
// positions spread over the context, as the engine passes them).
double plan_cost(int blocks, int Hk, int HD, int n_ctx, int tps, int sms) {
  const bool split = tps < ceil_div(n_ctx, BN);
  const double cta_cost = kItemCost + (split ? kSplitItemCost : 0.0);
  double total = 0.0;
  int64_t items_all = 0;
  int max_item = 0;
  for (int b = 0; b < blocks; ++b) {
    const int kt = std::max(1, ceil_div((int64_t(b) + 1) * n_ctx / blocks, BN));
    const int items = ceil_div(kt, tps);
    total += kt + items * cta_cost;
    items_all += items;
    max_item = std::max(max_item, std::min(kt, tps));
  }
  total *= Hk;
  const double combine = split ? double(items_all) * Hk * NQ * BM * (HD * 4 + 8) / 14.3e6 : 0.0;
  return total / sms + 0.5 * (max_item + cta_cost) + combine;
}

// Key-split plan: the tiles-per-split with the smallest estimated makespan (no split
// included).  Plans are cached per shape.
SplitPlan plan_splits(int M, int Hq, int Hk, int HD, int n_ctx) {
  struct Key {
    int M, Hq, Hk, HD, n_ctx, sms;
  };
  static std::mutex mu;
  static std::vector<std::pair<Key, SplitPlan>> cache;
  const int sms = num_sms();
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& e : cache)
      if (e.first.M == M && e.first.Hq == Hq && e.first.Hk == Hk && e.first.HD == HD &&
          e.first.n_ctx == n_ctx && e.first.sms == sms)
        return e.second;
  }
  const int T = BM / (Hq / Hk);
  SplitPlan p;
  p.blocks = ceil_div(M, NQ * T);
  const int max_kt = ceil_div(n_ctx, BN);
  const double unsplit = plan_cost(p.blocks, Hk, HD, n_ctx, max_kt, sms);
  int best_tps = max_kt;
  double best = unsplit;
  // at most 32 splits: the combine gives each split one lane
  for (int tps = std::max(2, ceil_div(max_kt, 32)); tps < max_kt; tps = tps < 8 ? tps + 1 : tps + tps / 4) {
    const double c = plan_cost(p.blocks, Hk, HD, n_ctx, tps, sms);
    if (c < best) {
      best = c;
      best_tps = tps;
    }
  }
  // split only when the estimate promises at least 10 %
  if (best > 0.90 * unsplit) best_tps = max_kt;
  p.tps = best_tps;
  p.max_splits = ceil_div(max_kt, p.tps);
  p.bytes = p.max_splits > 1 ? int64_t(p.blocks) * Hk * p.max_splits * NQ * BM * (int64_t(HD) * 4 + 8) : 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() < 256) cache.push_back({Key{M, Hq, Hk, HD, n_ctx, sms}, p});
  return p;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// [H][n_ctx][HD] bf16 cache as a 3-D map, box = 64 x 128 keys x 1 head (keys past n_ctx read 0)
int make_cache_map(CUtensorMap* map, const void* ptr, int H, int n_ctx, int HD) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled unavailable");
    return CKV_ERR_CUDA;
  }
  cuuint64_t dims[3] = {cuuint64_t(HD), cuuint64_t(n_ctx), cuuint64_t(H)};
  cuuint64_t strides[2] = {cuuint64_t(HD) * 2, cuuint64_t(n_ctx) * HD * 2};
  cuuint32_t box[3] = {64, BN, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (cache) failed (%d)", int(r));
    return CKV_ERR_CUDA;
  }
  return CKV_OK;
}

// q [M][Hq][HD] as a 3-D map (HD, Hq, M), box = 64 x G heads x T tokens: one box is the
// 64-column half of a packed Q tile, rows (token, head) token-major; tokens past M read 0
int make_q_map(CUtensorMap* map, const void* ptr, int M, int Hq, int G, int T, int HD) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled unavailable");
    return CKV_ERR_CUDA;
  }
  cuuint64_t dims[3] = {cuuint64_t(HD), cuuint64_t(Hq), cuuint64_t(M)};
  cuuint64_t strides[2] = {cuuint64_t(HD) * 2, cuuint64_t(Hq) * HD * 2};
  cuuint32_t box[3] = {64, cuuint32_t(G), cuuint32_t(T)};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (q) failed (%d)", int(r));
    return CKV_ERR_CUDA;
  }
  return CKV_OK;
}

// ---------------------------------------------------------------------------------
// One query token (decode): split-KV on CUDA cores.  The tensor-core kernel would fill
// a 128-row Q tile with G rows; here a CTA takes one KV head and one 64-key chunk for
// the G query heads of that head.  The chunk's K and V rows come into shared memory by
// coalesced loads, all in flight at once; each thread scores one key for up to half of
// the heads, a warp per head turns the scores into exponentials relative to the
// chunk's max, and each thread then accumulates one output column over the keys.  Chunks past the
// query's position write nothing; the combine merges the chunks up to it, so one grid
// (sized for n_ctx) serves every position, as a replayed CUDA graph needs.
constexpr int kDecKeys = 64;

inline int dec_chunks(int n_ctx) { return ceil_div(n_ctx, kDecKeys); }
inline int64_t dec_bytes(int Hq, int HD, int n_ctx) {
  return int64_t(dec_chunks(n_ctx)) * Hq * (int64_t(HD) * 4 + 8);
}

// scores of key `kk` of the chunk for heads [G0, G1) into s_p (log2 domain)
template <int HD, int G0, int G1, int KROW, int G>
__device__ __forceinline__ void decode_scores(const uint16_t (*s_k)[KROW], const float (*s_q)[HD],
                                              float (*s_p)[kDecKeys], int kk, bool visible, float scale_log2) {
  float acc[G1 - G0 > 0 ? G1 - G0 : 1];
#pragma unroll
  for (int g = 0; g < G1 - G0; ++g) acc[g] = 0.f;
#pragma unroll 4
  for (int ch = 0; ch < HD / 8; ++ch) {
    const uint4 kv = *reinterpret_cast<const uint4*>(&s_k[kk][ch * 8]);
    const uint32_t* kw = reinterpret_cast<const uint32_t*>(&kv);
    float kf[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      kf[2 * e] = lo_bf(kw[e]);
      kf[2 * e + 1] = hi_bf(kw[e]);
    }
#pragma unroll
    for (int g = 0; g < G1 - G0; ++g) {
      const float4 qa = *reinterpret_cast<const float4*>(&s_q[G0 + g][ch * 8]);
      const float4 qb = *reinterpret_cast<const float4*>(&s_q[G0 + g][ch * 8 + 4]);
      acc[g] = fmaf(qa.x, kf[0], fmaf(qa.y, kf[1], fmaf(qa.z, kf[2], fmaf(qa.w, kf[3], acc[g]))));
      acc[g] = fmaf(qb.x, kf[4], fmaf(qb.y, kf[5], fmaf(qb.z, kf[6], fmaf(qb.w, kf[7], acc[g]))));
    }
  }
#pragma unroll
  for (int g = 0; g < G1 - G0; ++g) s_p[G0 + g][kk] = visible ? acc[g] * scale_log2 : -INFINITY;
}

template <int HD, int G>
__global__ void __launch_bounds__(HD) decode_attention_kernel(
    const uint16_t* __restrict__ q, const uint16_t* __restrict__ kc, const uint16_t* __restrict__ vc,
    const int32_t* __restrict__ positions, int Hk, int n_ctx, float scale_log2, float* __restrict__ part_o,
    float2* __restrict__ part_ml) {
  // K rows padded by 16 bytes so that eight lanes reading eight rows hit distinct banks
  constexpr int kKRow = HD + 8;
  __shared__ __align__(16) uint16_t s_k[kDecKeys][kKRow];
  __shared__ __align__(16) uint16_t s_v[kDecKeys][HD];
  __shared__ __align__(16) float s_q[G][HD];
  __shared__ __align__(16) float s_p[G][kDecKeys];
  __shared__ float s_ml[G][2];
  const int c = blockIdx.x, hk = blockIdx.y;
  const int Hq = G * Hk;
  int pos = positions[0];
  if ((pos < 0 || pos >= n_ctx) && c == 0 && hk == 0 && threadIdx.x == 0)
    atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
  pos = pos < 0 ? 0 : (pos >= n_ctx ? n_ctx - 1 : pos);
  const int key0 = c * kDecKeys;
  if (key0 > pos) return;  // nothing visible in this chunk: the combine skips it
  const int t = threadIdx.x;
  const int n_keys = min(kDecKeys, pos + 1 - key0);
  // the chunk's K and V rows (zeros past the last visible key), all loads in flight at once
  {
    constexpr int kPer = kDecKeys / 8;  // 16-byte vectors per thread, of K and of V
    const uint4* kg = reinterpret_cast<const uint4*>(kc + (int64_t(hk) * n_ctx + key0) * HD);
    const uint4* vg = reinterpret_cast<const uint4*>(vc + (int64_t(hk) * n_ctx + key0) * HD);
    uint4 kv[kPer], vv[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int idx = t + HD * i, row = idx / (HD / 8);
      kv[i] = row < n_keys ? __ldg(kg + idx) : make_uint4(0u, 0u, 0u, 0u);
      vv[i] = row < n_keys ? __ldg(vg + idx) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) s_q[g][t] = bf2f(q[int64_t(hk * G + g) * HD + t]);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int idx = t + HD * i, row = idx / (HD / 8), ch = idx % (HD / 8);
      *reinterpret_cast<uint4*>(&s_k[row][ch * 8]) = kv[i];
      *reinterpret_cast<uint4*>(&s_v[row][ch * 8]) = vv[i];
    }
  }
  __syncthreads();
  // scores: with HD = 128 two threads per key, the first half of the heads and the rest
  // (a warp-uniform split: warps 0-1 and 2-3); with HD = 64 one thread per key
  {
    const int kk = t % kDecKeys;
    const bool vis = kk < n_keys;
    if constexpr (HD / kDecKeys == 2) {
      if (t < kDecKeys)
        decode_scores<HD, 0, G / 2, kKRow, G>(s_k, s_q, s_p, kk, vis, scale_log2);
      else
        decode_scores<HD, G / 2, G, kKRow, G>(s_k, s_q, s_p, kk, vis, scale_log2);
    } else {
      decode_scores<HD, 0, G, kKRow, G>(s_k, s_q, s_p, kk, vis, scale_log2);
    }
  }
  __syncthreads();
  // per head: chunk max, exponentials, sum (one warp per head)
  const int warp = t >> 5, lane = t & 31;
  for (int g = warp; g < G; g += HD / 32) {
    const float a = s_p[g][lane], b = s_p[g][lane + 32];
    float mx = fmaxf(a, b);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float pa = exp2f(a - mx), pb = exp2f(b - mx);  // key0 <= pos: mx is finite
    s_p[g][lane] = pa;
    s_p[g][lane + 32] = pb;
    float sum = pa + pb;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      s_ml[g][0] = mx;
      s_ml[g][1] = sum;
    }
  }
  __syncthreads();
  // P V: thread t owns output column t for every head (rows past the visible keys are 0);
  // P is read four keys at a time
  float o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) o[g] = 0.f;
#pragma unroll 2
  for (int j = 0; j < kDecKeys; j += 4) {
    const float v0 = bf2f(s_v[j][t]), v1 = bf2f(s_v[j + 1][t]), v2 = bf2f(s_v[j + 2][t]),
                v3 = bf2f(s_v[j + 3][t]);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float4 p4 = *reinterpret_cast<const float4*>(&s_p[g][j]);
      o[g] = fmaf(p4.x, v0, fmaf(p4.y, v1, fmaf(p4.z, v2, fmaf(p4.w, v3, o[g]))));
    }
  }
  const int64_t row0 = int64_t(c) * Hq + hk * G;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    part_o[(row0 + g) * HD + t] = o[g];
    if (t == 0) part_ml[row0 + g] = make_float2(s_ml[g][0], s_ml[g][1]);
  }
}

// Merge the chunks of the decode kernel: out = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c.
// A CTA takes one query head and 32 output columns; its 32 warps take chunks w, w + 32,
// ... (one column per lane, loads coalesced), and meet in shared memory.
constexpr int kDecCombineWarps = 32;
template <int HD>
__global__ void __launch_bounds__(kDecCombineWarps * 32) decode_combine_kernel(
    const int32_t* __restrict__ positions, uint16_t* __restrict__ out, int Hq, int n_ctx,
    const float* __restrict__ part_o, const float2* __restrict__ part_ml) {
  __shared__ float s_red[kDecCombineWarps];
  __shared__ float s_acc[kDecCombineWarps][33];
  __shared__ float s_l[kDecCombineWarps];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int hq = blockIdx.x, col = blockIdx.y * 32 + lane;
  int pos = positions[0];
  pos = pos < 0 ? 0 : (pos >= n_ctx ? n_ctx - 1 : pos);
  const int n = pos / kDecKeys + 1;  // chunks that hold visible keys
  float mx = -INFINITY;
  for (int c = threadIdx.x; c < n; c += kDecCombineWarps * 32) mx = fmaxf(mx, part_ml[int64_t(c) * Hq + hq].x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_red[wp] = mx;
  __syncthreads();
  mx = s_red[0];
#pragma unroll
  for (int i = 1; i < kDecCombineWarps; ++i) mx = fmaxf(mx, s_red[i]);
  float L = 0.f, acc = 0.f;
#pragma unroll 4
  for (int c = wp; c < n; c += kDecCombineWarps) {
    const float2 ml = part_ml[int64_t(c) * Hq + hq];
    const float wgt = exp2f(ml.x - mx);
    L = fmaf(wgt, ml.y, L);
    acc = fmaf(wgt, part_o[(int64_t(c) * Hq + hq) * HD + col], acc);
  }
  s_acc[wp][lane] = acc;
  if (lane == 0) s_l[wp] = L;
  __syncthreads();
  if (wp == 0) {
    float a = 0.f, l = 0.f;
#pragma unroll 8
    for (int k = 0; k < kDecCombineWarps; ++k) {
      a += s_acc[k][lane];
      l += s_l[k];
    }
    out[int64_t(hq) * HD + col] = f2bf(l > 0.f ? a / l : 0.f);
  }
}

template <int HD, int G>
void launch_decode_g(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* positions,
                     int Hk, int n_ctx, float sl2, float* part_o, float2* part_ml, cudaStream_t stream) {
  decode_attention_kernel<HD, G><<<dim3(dec_chunks(n_ctx), Hk), HD, 0, stream>>>(q, kc, vc, positions, Hk, n_ctx,
                                                                                sl2, part_o, part_ml);
}

// G values with a compiled decode kernel (Qwen2 shapes: 1 MHA, 2 / 4 / 5 / 6 / 7 / 8 GQA, 16)
inline bool decode_g_ok(int G) {
  return G == 1 || G == 2 || G == 4 || G == 5 || G == 6 || G == 7 || G == 8 || G == 16;
}

template <int HD>
int launch_decode(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* positions,
                  uint16_t* out, int Hq, int Hk, int n_ctx, float scale, void* workspace, cudaStream_t stream) {
  float* part_o = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kSchedBytes);
  float2* part_ml = reinterpret_cast<float2*>(part_o + int64_t(dec_chunks(n_ctx)) * Hq * HD);
  const float sl2 = scale * 1.4426950408889634f;
  switch (Hq / Hk) {
    case 1: launch_decode_g<HD, 1>(q, kc, vc, positions, Hk, n_ctx, sl2, part_o, part_ml, stream); break;
    case 2: launch_decode_g<HD, 2>(q, kc, vc, positions, Hk, n_ctx, sl2, part_o, part_ml, stream); break;
    case 4: launch_decode_g<HD, 4>(q, kc, vc, positions, Hk, n_ctx, sl2, part_o, part_ml, stream); break;
    case 5: launch_decode_g<HD, 5>(q, kc, vc, positions, Hk, n_ctx, sl2, part_o, part_ml, stream); break;
    case 6: launch_decode_g<HD, 6>(q, kc, vc, positions, Hk, n_ctx, sl2, part_o, part_ml, stream); break;
    case 7: launch_decode_g<HD, 7>(q, kc, vc, positions, Hk, n_ctx, sl2, part_o, part_ml, stream); break;
    case 8: launch_decode_g<HD, 8>(q, kc, vc, positions, Hk, n_ctx, sl2, part_o, part_ml, stream); break;
    case 16: launch_decode_g<HD, 16>(q, kc, vc, positions, Hk, n_ctx, sl2, part_o, part_ml, stream); break;
    default:
      set_error("ckv_attention(decode): %d query heads per KV head", Hq / Hk);
      return CKV_ERR_UNSUPPORTED;
  }
  CKV_LAUNCH_CHECK("ckv_attention(decode)");
  decode_combine_kernel<HD><<<dim3(Hq, HD / 32), kDecCombineWarps * 32, 0, stream>>>(positions, out, Hq, n_ctx,
                                                                                      part_o, part_ml);
  CKV_LAUNCH_CHECK("ckv_attention(decode combine)");
  return CKV_OK;
}

// decode path: one query token, a G with a compiled decode kernel, and room for
// the chunk partials after the scheduler words
inline bool use_decode(int M, int Hq, int Hk, int HD, int n_ctx, int64_t ws_bytes) {
  return M == 1 && decode_g_ok(Hq / Hk) && ws_bytes >= kSchedBytes + dec_bytes(Hq, HD, n_ctx);
}

template <int HD>
int launch(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* positions, uint16_t* out,
           int M, int Hq, int Hk, int n_ctx, float scale, void* workspace, int64_t ws_bytes,
           cudaStream_t stream) {
  if (use_decode(M, Hq, Hk, HD, n_ctx, ws_bytes))
    return launch_decode<HD>(q, kc, vc, positions, out, Hq, Hk, n_ctx, scale, workspace, stream);
  CUtensorMap mk, mv, mq;
  if (int rc = make_cache_map(&mk, kc, Hk, n_ctx, HD)) return rc;
  if (int rc = make_cache_map(&mv, vc, Hk, n_ctx, HD)) return rc;
  if (int rc = make_q_map(&mq, q, M, Hq, Hq / Hk, BM / (Hq / Hk), HD)) return rc;
  auto kern = attention_tc_kernel<HD>;
  if (int rc = set_smem_limit(reinterpret_cast<const void*>(kern), Cfg<HD>::SMEM)) return rc;
  SplitPlan p = plan_splits(M, Hq, Hk, HD, n_ctx);
  // scheduler words when the workspace has room for them; split partials when it has
  // room for those too
  unsigned* sched = ws_bytes >= kSchedBytes ? static_cast<unsigned*>(workspace) : nullptr;
  if (p.max_splits > 1 && ws_bytes < kSchedBytes + p.bytes) {  // no room: one split
    p.tps = ceil_div(n_ctx, BN);
    p.max_splits = 1;
  }
  float* part_o = p.max_splits > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kSchedBytes)
                                   : nullptr;
  float2* part_ml = p.max_splits > 1
                        ? reinterpret_cast<float2*>(part_o + int64_t(p.blocks) * Hk * p.max_splits * NQ * BM * HD)
                        : nullptr;
  const float sl2 = scale * 1.4426950408889634f;
  const int64_t n_slots = int64_t(p.blocks) * Hk * p.max_splits;
  CKV_REQUIRE(n_slots < (int64_t(1) << 31) - 4 * 1024 * 1024, "ckv_attention: too many work items");
  const int grid = int(std::min<int64_t>(n_slots, num_sms()));
  launch_pdl(kern, dim3(grid), dim3(kThreads), Cfg<HD>::SMEM, stream, mk, mv, mq, positions, out, M, Hq, Hk,
             n_ctx, sl2, p.tps, p.max_splits, p.blocks, sched, part_o, part_ml);
  CKV_LAUNCH_CHECK("ckv_attention");
  if (p.max_splits > 1) {
    launch_pdl(attention_combine_kernel<HD>, dim3(p.blocks * (NQ * BM / (kCombineWarps * kCombineRows)), Hk),
               dim3(kCombineWarps * 32), 0, stream, positions, out, M, Hq, Hk, n_ctx, p.tps, p.max_splits,
               static_cast<const float*>(part_o), static_cast<const float2*>(part_ml));
    CKV_LAUNCH_CHECK("ckv_attention(combine)");
  }
  return CKV_OK;
}

}  // namespace
}  // namespace ckv

using namespace ckv;

extern "C" int64_t ckv_attention_workspace_size(int m, int n_q_heads, int n_kv_heads, int head_dim,
                                                int n_ctx) {
  if (m <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0 || n_ctx <= 0 ||
      (head_dim != 64 && head_dim != 128) || n_q_heads / n_kv_heads > BM)
    return 0;
  if (m == 1 && decode_g_ok(n_q_heads / n_kv_heads)) return kSchedBytes + dec_bytes(n_q_heads, head_dim, n_ctx);
  return kSchedBytes + plan_splits(m, n_q_heads, n_kv_heads, head_dim, n_ctx).bytes;
}

extern "C" int ckv_attention_launches(int m, int n_q_heads, int n_kv_heads, int head_dim, int n_ctx,
                                      int64_t workspace_bytes) {
  if (m <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0 || n_ctx <= 0 ||
      (head_dim != 64 && head_dim != 128) || n_q_heads / n_kv_heads > BM)
    return 0;
  if (use_decode(m, n_q_heads, n_kv_heads, head_dim, n_ctx, workspace_bytes)) return 2;  // + its combine
  const SplitPlan p = plan_splits(m, n_q_heads, n_kv_heads, head_dim, n_ctx);
  return p.max_splits > 1 && workspace_bytes >= kSchedBytes + p.bytes ? 2 : 1;  // + the combine kernel
}

extern "C" int ckv_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                             const int32_t* positions, uint16_t* out, int m, int n_q_heads, int n_kv_heads,
                             int head_dim, int n_ctx, float scale, void* workspace,
                             int64_t workspace_bytes, ckv_stream_t stream) {
  CKV_REQUIRE(q && k_cache && v_cache && positions && out, "ckv_attention: null pointer");
  CKV_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out),
              "ckv_attention: tensors must be 16-byte aligned");
  CKV_REQUIRE(n_kv_heads > 0 && n_q_heads % n_kv_heads == 0,
              "ckv_attention: n_q_heads %d not a multiple of n_kv_heads %d", n_q_heads, n_kv_heads);
  CKV_REQUIRE(n_q_heads / n_kv_heads <= BM, "ckv_attention: more than %d query heads per KV head", BM);
  CKV_REQUIRE(n_kv_heads <= 65535 && n_ctx > 0 && m >= 0, "ckv_attention: bad sizes");
  if (m == 0) return CKV_OK;
  CKV_REQUIRE(workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 15u) == 0,
              "ckv_attention: workspace must be 16-byte aligned");
  if (head_dim == 128)
    return launch<128>(q, k_cache, v_cache, positions, out, m, n_q_heads, n_kv_heads, n_ctx, scale,
                       workspace, workspace_bytes, as_stream(stream));
  if (head_dim == 64)
    return launch<64>(q, k_cache, v_cache, positions, out, m, n_q_heads, n_kv_heads, n_ctx, scale,
                      workspace, workspace_bytes, as_stream(stream));
  set_error("ckv_attention: head_dim %d (64 or 128)", head_dim);
  return CKV_ERR_UNSUPPORTED;
}
