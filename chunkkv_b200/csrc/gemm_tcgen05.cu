// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), with the
// epilogues of the recompute layers fused in:
//   EPI_STORE  out = bf16(x W^T (+ bias))                      nn.Linear
//   EPI_RESID  h   = bf16(h + bf16(x W^T))                      torch_engine.py:72-73
//   EPI_SWIGLU out = bf16(silu(bf16(g)) * bf16(u))              Qwen2MLP gate/up
//   EPI_QKV    q/k/v = bf16(x W^T + b), RoPE at positions on q,k (torch_engine.py:61-66),
//              k/v written straight into the blended cache       (torch_engine.py:155-156)
//
// D = A B^T with A = x [M][K] and B = W [N][K], both K-major.  One persistent CTA
// per SM, 10 warps:
//   warp 0      TMA producer (one thread): A 128x64 and B 256x64 tiles, 128B swizzle,
//               4-stage ring guarded by full/empty mbarriers;
//   warp 1      TMEM owner + MMA issuer (one thread): tcgen05.mma kind::f16,
//               M=128 N=256 K=16 per instruction, fp32 accumulators in TMEM;
//   warps 2..9  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows; warps w and w+4 take the two halves of the
//               tile's columns), fused math, stores.
// Two 256-column accumulators (all 512 TMEM columns) let the epilogue of one tile
// overlap the main loop of the next.  Tiles are visited M-fastest so CTAs that
// run together share the same weight tile through L2.
//
// Every mbarrier wait is bounded (ckv::mbar_wait); a wait that runs out sets
// CKV_DEV_ERR_WAIT_TIMEOUT, the CTA drains what it issued and frees its TMEM.
#include <algorithm>
#include <mutex>

#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(gemm)

namespace ckv {
namespace {

constexpr int BM = 128, BK = 64, UMMA_K = 16;
// warp 0 TMA, warp 1 MMA, warps 2..9 epilogue: two warps per TMEM lane quadrant, each
// taking one half of the tile's columns
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t A_BYTES = BM * BK * 2;  // 16 KiB
constexpr uint32_t TMEM_COLS = 512;        // two accumulators of up to 256 columns

// N-tile width: 256, or 224 / 208 when that fills the SMs better (e.g. 3584 columns at
// M = 938: 144 tiles of 208 in one wave instead of 112 of 256 on 148 SMs).
template <int BN, int ST = 4>
struct GCfg {
  static_assert(BN % 16 == 0 && BN <= 256, "BN");
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = ST;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
  static_assert(SMEM_BYTES <= 227 * 1024, "stages do not fit in shared memory");
  static constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN);
};

enum Epi { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKV = 3, EPI_PARTIAL = 4 };

struct EpiParams {
  const uint16_t* bias;  // by absolute column of the full weight (STORE optional, QKV)
  uint16_t* out;         // STORE out, RESID h, SWIGLU out
  int64_t ldo;
  const int32_t* positions;
  const float2* rope;
  int rope_max_pos;
  int col_begin;
  int n_q_heads, n_kv_heads;
  uint16_t* q_out;
  uint16_t* k_cache;
  uint16_t* v_cache;
  int n_ctx;
  uint16_t* k_compact;
  uint16_t* v_compact;
  // EPI_PARTIAL (tensor parallel): the tile is stored like EPI_STORE (this rank's partial
  // rows, read by the other ranks over NVLink); the last CTA to finish then adds 1 to
  // every rank's counter for this rank.
  const uint64_t* push_flag;  // [ranks] address of each rank's uint32 counters [ranks]
  unsigned* push_ticket;      // this rank's CTA ticket (left at 0)
  int push_rank, push_ranks;
};

__device__ __forceinline__ void store8(uint16_t* dst, const float* v) {
  uint4 w;
  w.x = pack_bf2(v[0], v[1]);
  w.y = pack_bf2(v[2], v[3]);
  w.z = pack_bf2(v[4], v[5]);
  w.w = pack_bf2(v[6], v[7]);
  *reinterpret_cast<uint4*>(dst) = w;
}

// ---- epilogues: one thread = one tile row; all lanes execute the TMEM loads.  `part`
// (0 or 1) selects which half of the tile's 32-column chunks (or heads) this warp does.
template <int BN>
__device__ __forceinline__ int chunk_lo(int part) {
  constexpr int n = (BN + 31) / 32;
  return part == 0 ? 0 : 32 * ((n + 1) / 2);
}
template <int BN>
__device__ __forceinline__ int chunk_hi(int part) {
  constexpr int n = (BN + 31) / 32;
  return part == 0 ? 32 * ((n + 1) / 2) : 32 * n;
}

template <int BN>
__device__ __forceinline__ void epi_store(uint32_t tacc, int row, int M, int n0, int N,
                                          const EpiParams& ep, int part) {
#pragma unroll 1
  for (int c = chunk_lo<BN>(part); c < chunk_hi<BN>(part); c += 32) {
    float v[32];
    tmem_ld32(tacc + c, v);
    if (row >= M) continue;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int col = n0 + c + g * 8;
      if (c + g * 8 >= BN || col >= N) continue;  // BN may end mid-chunk (208 = 6.5 x 32)
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o[e] = v[g * 8 + e];
        if (ep.bias) o[e] = __fadd_rn(o[e], bf2f(ep.bias[col + e]));
      }
      store8(ep.out + int64_t(row) * ep.ldo + col, o);
    }
  }
}

template <int BN>
__device__ __forceinline__ void epi_resid(uint32_t tacc, int row, int M, int n0, int N,
                                          const EpiParams& ep, int part) {
  constexpr int kChunks = ((BN + 31) / 32 + 1) / 2;  // 32-column chunks per part (<= 4)
  const int c_lo = chunk_lo<BN>(part), c_hi = chunk_hi<BN>(part);
  // every residual vector of this thread's part of the row is requested before the first
  // TMEM load, so one global round trip serves the whole part
  uint4 hv[kChunks][4];
#pragma unroll
  for (int ci = 0; ci < kChunks; ++ci) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int c = c_lo + 32 * ci;
      const int col = n0 + c + g * 8;
      hv[ci][g] = make_uint4(0u, 0u, 0u, 0u);
      if (row < M && c < c_hi && c + g * 8 < BN && col < N)
        hv[ci][g] = *reinterpret_cast<const uint4*>(ep.out + int64_t(row) * ep.ldo + col);
    }
  }
#pragma unroll
  for (int ci = 0; ci < kChunks; ++ci) {
    const int c = c_lo + 32 * ci;
    if (c >= c_hi) break;  // warp-uniform
    float v[32];
    tmem_ld32(tacc + c, v);
    if (row >= M) continue;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int col = n0 + c + g * 8;
      if (c + g * 8 >= BN || col >= N) continue;
      const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hv[ci][g]);
      float o[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        o[2 * e] = __fadd_rn(lo_bf(hw[e]), bf16_round(v[g * 8 + 2 * e]));
        o[2 * e + 1] = __fadd_rn(hi_bf(hw[e]), bf16_round(v[g * 8 + 2 * e + 1]));
      }
      store8(ep.out + int64_t(row) * ep.ldo + col, o);
    }
  }
}

// Tile = 128 gate columns then the 128 matching up columns (interleaved weight).
template <int BN>
__device__ __forceinline__ void epi_swiglu(uint32_t tacc, int row, int M, int n0, int N,
                                           const EpiParams& ep, int part) {
  const int out0 = n0 / 2;
#pragma unroll 1
  for (int c = chunk_lo<BN / 2>(part); c < chunk_hi<BN / 2>(part); c += 32) {
    float g[32], u[32];
    tmem_ld32(tacc + c, g);
    tmem_ld32(tacc + BN / 2 + c, u);
    if (row >= M || n0 >= N) continue;
    float o[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float gb = bf16_round(g[j]);
      const float s = bf16_round(__fdiv_rn(gb, __fadd_rn(1.0f, expf(-gb))));
      o[j] = __fmul_rn(s, bf16_round(u[j]));
    }
    uint16_t* dst = ep.out + int64_t(row) * ep.ldo + out0 + c;
#pragma unroll
    for (int q = 0; q < 4; ++q) store8(dst + q * 8, o + q * 8);
  }
}

template <int BN, int HD>
__device__ __forceinline__ void epi_qkv(uint32_t tacc, int row, int M, int n0, int N,
                                        const EpiParams& ep, int part) {
  constexpr int HALF = HD / 2;
  const int Hq = ep.n_q_heads, Hk = ep.n_kv_heads;
  int pos = 0;
  bool ok = row < M;
  if (ok) {
    pos = ep.positions[row];
    const bool bad = pos < 0 || pos >= ep.rope_max_pos || (ep.k_cache && pos >= ep.n_ctx);
    if (bad) {
      atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
      ok = false;
    }
  }
  constexpr int kHeads = BN / HD;  // heads per tile, split between the two parts
#pragma unroll 1
  for (int hh = part * ((kHeads + 1) / 2); hh < (part == 0 ? (kHeads + 1) / 2 : kHeads); ++hh) {
    if (n0 + hh * HD >= N) break;  // warp-uniform
    const int gcol = ep.col_begin + n0 + hh * HD;
    const int head = gcol / HD;
    const uint32_t tcol = tacc + hh * HD;
    if (head < Hq + Hk) {
      uint16_t* dst;
      if (head < Hq) {
        dst = ep.q_out + int64_t(row) * (Hq * HD) + head * HD;
      } else if (ep.k_cache) {
        dst = ep.k_cache + (int64_t(head - Hq) * ep.n_ctx + pos) * HD;
      } else {
        dst = ep.k_compact + int64_t(row) * (Hk * HD) + (head - Hq) * HD;
      }
      const float2* cs = ep.rope + int64_t(pos) * HALF;
#pragma unroll 1
      for (int c = 0; c < HALF; c += 32) {
        float x1[32], x2[32];
        tmem_ld32(tcol + c, x1);
        tmem_ld32(tcol + HALF + c, x2);
        if (!ok) continue;
        // (cos, sin) of the 32 rotary pairs of this chunk: 16 x 16-byte loads of the row
        float4 t[16];
        const float4* cs4 = reinterpret_cast<const float4*>(cs + c);
#pragma unroll
        for (int q4 = 0; q4 < 16; ++q4) t[q4] = __ldg(cs4 + q4);
        float o1[32], o2[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float a = bf16_round(__fadd_rn(x1[j], bf2f(ep.bias[gcol + c + j])));
          const float b = bf16_round(__fadd_rn(x2[j], bf2f(ep.bias[gcol + HALF + c + j])));
          const float rc = (j & 1) ? t[j >> 1].z : t[j >> 1].x;
          const float rs = (j & 1) ? t[j >> 1].w : t[j >> 1].y;
          o1[j] = __fsub_rn(__fmul_rn(a, rc), __fmul_rn(b, rs));
          o2[j] = __fadd_rn(__fmul_rn(a, rs), __fmul_rn(b, rc));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          store8(dst + c + q * 8, o1 + q * 8);
          store8(dst + HALF + c + q * 8, o2 + q * 8);
        }
      }
    } else {
      const int hv = head - Hq - Hk;
      uint16_t* dst = ep.v_cache ? ep.v_cache + (int64_t(hv) * ep.n_ctx + pos) * HD
                                 : ep.v_compact + int64_t(row) * (Hk * HD) + hv * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float x[32];
        tmem_ld32(tcol + c, x);
        if (!ok) continue;
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = __fadd_rn(x[j], bf2f(ep.bias[gcol + c + j]));
#pragma unroll
        for (int q = 0; q < 4; ++q) store8(dst + c + q * 8, x + q * 8);
      }
    }
  }
}

template <int EPI, int HD, int BN>
__device__ __forceinline__ void run_epilogue(uint32_t tacc, int row, int M, int n0, int N,
                                             const EpiParams& ep, int part) {
  if constexpr (EPI == EPI_STORE) epi_store<BN>(tacc, row, M, n0, N, ep, part);
  else if constexpr (EPI == EPI_RESID) epi_resid<BN>(tacc, row, M, n0, N, ep, part);
  else if constexpr (EPI == EPI_SWIGLU) epi_swiglu<BN>(tacc, row, M, n0, N, ep, part);
  else if constexpr (EPI == EPI_PARTIAL) epi_store<BN>(tacc, row, M, n0, N, ep, part);
  else epi_qkv<BN, HD>(tacc, row, M, n0, N, ep, part);
}

// Bounded wait that ignores the abort flag (used only while draining).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitLimitNs) break;
}

template <int EPI, int HD, int BN, int ST>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                int M, int N, int K, EpiParams ep) {
  using C = GCfg<BN, ST>;
  constexpr uint32_t B_BYTES = C::B_BYTES, STAGE_BYTES = C::STAGE_BYTES, IDESC = C::IDESC;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
    fence_async_smem();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The weights are not written by the kernels before, so the weight tiles of the first
  // stages are requested before the dependent-launch wait and arrive while the previous
  // kernel ends; A and everything the epilogue touches wait for it.
  int pre = 0;
  if (warp == 0 && lane == 0 && int(blockIdx.x) < num_tiles) {
    pre = min(STAGES, num_kb);
    const int nt0 = int(blockIdx.x) / m_tiles;
    for (int kb = 0; kb < pre; ++kb) {
      mbar_expect_tx(&full[kb], STAGE_BYTES);
      tma_load_2d(sB + kb * B_BYTES, &tmB, kb * BK, nt0 * BN, &full[kb]);
    }
  }
  pdl_wait();
  pdl_launch_next();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mt = tile % m_tiles, nt = tile / m_tiles;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (it < pre) {  // weight tile already requested: the activation tile joins it
            tma_load_2d(sA + s * A_BYTES, &tmA, kb * BK, mt * BM, &full[s]);
            continue;
          }
          if (!mbar_wait(&empty[s], ph ^ 1, abort, &g_err_word)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmA, kb * BK, mt * BM, &full[s]);
          tma_load_2d(sB + s * B_BYTES, &tmB, kb * BK, nt * BN, &full[s]);
        }
      }
      if (!ok)  // let the copies already issued land before the CTA goes away
        for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
          drain_wait(&full[j % STAGES], (j / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++tcount) {
        const int acc = tcount & 1;
        const uint32_t use = tcount >> 1;
        if (!mbar_wait(&tempty[acc], (use & 1) ^ 1, abort, &g_err_word)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;  // accumulators at columns 0 and 256
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort, &g_err_word)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * A_BYTES);
          const uint32_t b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t ad = umma_desc_sw128(a0 + k * UMMA_K * 2);
            const uint64_t bd = umma_desc_sw128(b0 + k * UMMA_K * 2);
            tc_mma_f16(d_tmem, ad, bd, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&tfull[acc]);
      }
      if (!ok) {  // wait for the MMAs already issued before TMEM is released
        tc_commit(drain);
        drain_wait(drain, 0);
      }
    }
  } else {
    const int sub = warp & 3;             // TMEM sub-partition this warp may access
    const int part = (warp - 2) / 4;      // which half of the tile's columns
    int tcount = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tcount) {
      const int acc = tcount & 1;
      const uint32_t use = tcount >> 1;
      if (!mbar_wait(&tfull[acc], use & 1, abort, &g_err_word)) break;
      tc_fence_after();
      const int mt = tile % m_tiles, nt = tile / m_tiles;
      const int row = mt * BM + sub * 32 + lane;
      const uint32_t tacc = tmem_base + (uint32_t(sub * 32) << 16) + acc * 256;
      run_epilogue<EPI, HD, BN>(tacc, row, M, nt * BN, N, ep, part);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  if constexpr (EPI == EPI_PARTIAL) __threadfence_system();  // this thread's rows first
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if constexpr (EPI == EPI_PARTIAL) {
    // the last CTA tells every rank that this rank's partial rows are all written
    if (threadIdx.x == 0) {
      const unsigned t = atomicAdd(ep.push_ticket, 1u);
      if (t == gridDim.x - 1) {
        __threadfence_system();
        for (int q = 0; q < ep.push_ranks; ++q)
          red_release_sys_add(reinterpret_cast<unsigned*>(ep.push_flag[q]) + ep.push_rank, 1u);
        *ep.push_ticket = 0u;
      }
    }
  }
}

// ---- the same GEMM on CTA pairs.  A cluster of two CTAs (the two SMs of a TPC) owns a
// 256 x BN tile: CTA r loads rows [128r, 128r + 128) of A and rows [r BN/2, (r+1) BN/2)
// of B into its own shared memory, and CTA 0 issues tcgen05.mma.cta_group::2 (M = 256),
// which reads both CTAs' operands and leaves rows 128r.. of the accumulator in CTA r's
// TMEM.  Per SM and k-step the shared memory takes 32 KiB of loads and serves 32 KiB to
// the tensor core, against 48 + 48 KiB for a one-SM 128 x 256 tile: the one-SM kernel's
// k-loop is bound by shared-memory bandwidth, this one by the tensor core.
//   full[s]    CTA 0 only: CTA 0's expect_tx for both CTAs' bytes; both CTAs' copies
//              complete on it (loads without multicast)
//   empty[s]   both CTAs: the pair MMA's commit arrives on both
//   tfull[a]   both CTAs: accumulator a is complete (commit to both)
//   tempty[a]  CTA 0 only: 2 x kEpiWarps arrivals, the peer's from across the pair
template <int BN, int ST>
struct PCfg {
  static constexpr int BNH = BN / 2;  // B rows per CTA
  static_assert(BN % 16 == 0 && BN <= 256 && BNH % 8 == 0, "BN");
  static constexpr uint32_t B_BYTES = BNH * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;  // one CTA's share of a stage
  static constexpr int STAGES = ST;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
  static_assert(SMEM_BYTES <= 227 * 1024, "stages do not fit in shared memory");
  static_assert(B_BYTES % 1024 == 0, "B stages must keep the 1024-byte swizzle alignment");
  static constexpr uint32_t IDESC = umma_idesc_bf16(2 * BM, BN);
};

template <int EPI, int HD, int BN, int ST>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     int M, int N, int K, EpiParams ep) {
  using C = PCfg<BN, ST>;
  constexpr uint32_t B_BYTES = C::B_BYTES, STAGE_BYTES = C::STAGE_BYTES, IDESC = C::IDESC;
  constexpr int STAGES = C::STAGES, BNH = C::BNH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int m_tiles = (M + 2 * BM - 1) / (2 * BM);
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
    fence_async_smem();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  // both CTAs' barriers are initialised before either CTA's copies or arrivals reach them
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the weight halves of the first stages go out before the dependent-launch wait (the
  // weights are not written by the kernels before); A waits for the previous kernel
  int pre = 0;
  if (warp == 0 && lane == 0 && pair < num_tiles) {
    pre = min(STAGES, num_kb);
    const int yb0 = (pair / m_tiles) * BN + int(rank) * BNH;
    for (int kb = 0; kb < pre; ++kb) {
      if (rank == 0) mbar_expect_tx(&full[kb], 2 * STAGE_BYTES);
      tma_load_2d_pair(sB + kb * B_BYTES, &tmB, kb * BK, yb0, cluster_smem_addr(&full[kb], 0));
    }
  }
  pdl_wait();
  pdl_launch_next();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += n_pairs) {
        const int mt = tile % m_tiles, nt = tile / m_tiles;
        const int ya = mt * 2 * BM + int(rank) * BM, yb = nt * BN + int(rank) * BNH;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const uint32_t bar = cluster_smem_addr(&full[s], 0);
          if (it < pre) {  // weight half already requested: the activation rows join it
            tma_load_2d_pair(sA + s * A_BYTES, &tmA, kb * BK, ya, bar);
            continue;
          }
          if (!mbar_wait(&empty[s], ph ^ 1, abort, &g_err_word)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_expect_tx(&full[s], 2 * STAGE_BYTES);
          tma_load_2d_pair(sA + s * A_BYTES, &tmA, kb * BK, ya, bar);
          tma_load_2d_pair(sB + s * B_BYTES, &tmB, kb * BK, yb, bar);
        }
      }
      // CTA 0 lets the copies already issued (its own and the peer's) land before the
      // pair goes away; the peer's copies complete on CTA 0's barriers, and the peer
      // stays resident until the cluster barrier at the end
      if (!ok && rank == 0)
        for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
          drain_wait(&full[j % STAGES], (j / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int it = 0, tcount = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += n_pairs, ++tcount) {
        const int acc = tcount & 1;
        const uint32_t use = tcount >> 1;
        if (!mbar_wait(&tempty[acc], (use & 1) ^ 1, abort, &g_err_word)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort, &g_err_word)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * A_BYTES);
          const uint32_t b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t ad = umma_desc_sw128(a0 + k * UMMA_K * 2);
            const uint64_t bd = umma_desc_sw128(b0 + k * UMMA_K * 2);
            tc_mma_f16_pair(d_tmem, ad, bd, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit_pair(&empty[s]);
        }
        if (ok) tc_commit_pair(&tfull[acc]);
      }
      if (!ok) {  // wait for the MMAs already issued before TMEM is released
        tc_commit_pair_local(drain);
        drain_wait(drain, 0);
      }
    }
  } else {
    const int sub = warp & 3;
    const int part = (warp - 2) / 4;
    const uint32_t tempty0[2] = {cluster_smem_addr(&tempty[0], 0), cluster_smem_addr(&tempty[1], 0)};
    int tcount = 0;
    for (int tile = pair; tile < num_tiles; tile += n_pairs, ++tcount) {
      const int acc = tcount & 1;
      const uint32_t use = tcount >> 1;
      if (!mbar_wait(&tfull[acc], use & 1, abort, &g_err_word)) break;
      tc_fence_after();
      const int mt = tile % m_tiles, nt = tile / m_tiles;
      const int row = mt * 2 * BM + int(rank) * BM + sub * 32 + lane;
      const uint32_t tacc = tmem_base + (uint32_t(sub * 32) << 16) + acc * 256;
      run_epilogue<EPI, HD, BN>(tacc, row, M, nt * BN, N, ep, part);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0[acc]);
    }
  }

  if constexpr (EPI == EPI_PARTIAL) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  // neither CTA leaves (or frees TMEM) while the other may still signal its barriers,
  // copy into its shared memory or run MMAs into its TMEM
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  if constexpr (EPI == EPI_PARTIAL) {
    if (threadIdx.x == 0) {
      const unsigned t = atomicAdd(ep.push_ticket, 1u);
      if (t == gridDim.x - 1) {
        __threadfence_system();
        for (int q = 0; q < ep.push_ranks; ++q)
          red_release_sys_add(reinterpret_cast<unsigned*>(ep.push_flag[q]) + ep.push_rank, 1u);
        *ep.push_ticket = 0u;
      }
    }
  }
}

// ---------------------------------------------------------------- host side
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
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Row-major bf16 [rows][k] (row stride ld elements), box = box_rows x 64.
int make_map(CUtensorMap* map, const void* ptr, int rows, int k, int64_t ld, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_error("cuTensorMapEncodeTiled unavailable (driver too old?)");
    return CKV_ERR_CUDA;
  }
  cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {cuuint32_t(BK), cuuint32_t(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) rows=%d k=%d ld=%lld", int(r), rows, k,
              (long long)ld);
    return CKV_ERR_CUDA;
  }
  return CKV_OK;
}

template <int EPI, int HD, int BN, int ST = 4>
int launch_bn(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, int M, int N, int K,
              const EpiParams& ep, cudaStream_t stream, const char* name) {
  CKV_REQUIRE(a && b, "%s: null operand", name);
  CKV_REQUIRE(M >= 0 && N > 0 && K > 0, "%s: bad sizes m=%d n=%d k=%d", name, M, N, K);
  CKV_REQUIRE(aligned16(a) && aligned16(b), "%s: operands must be 16-byte aligned", name);
  CKV_REQUIRE(K % 8 == 0 && lda % 8 == 0 && ldb % 8 == 0,
              "%s: k and row strides must be multiples of 8", name);
  CKV_REQUIRE(N % 16 == 0, "%s: n=%d must be a multiple of 16", name, N);
  if (M == 0) return CKV_OK;
  CUtensorMap ma, mb;
  if (int rc = make_map(&ma, a, M, K, lda, BM)) return rc;
  if (int rc = make_map(&mb, b, N, K, ldb, BN)) return rc;
  auto kern = gemm_kernel<EPI, HD, BN, ST>;
  if (int rc = set_smem_limit(reinterpret_cast<const void*>(kern), GCfg<BN, ST>::SMEM_BYTES)) return rc;
  const int tiles = ceil_div(M, BM) * ceil_div(N, BN);
  const int grid = std::min(tiles, num_sms());
  launch_pdl(kern, dim3(grid), dim3(kThreads), GCfg<BN, ST>::SMEM_BYTES, stream, ma, mb, M, N, K, ep);
  CKV_LAUNCH_CHECK(name);
  return CKV_OK;
}

// CTA pairs of a pair kernel that are resident at once (queried once per kernel and
// device); 0 when the query fails.
int resident_pairs(const void* kern, int smem) {
  struct Entry {
    const void* kern;
    int dev, pairs;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int n_cache = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n_cache; ++i)
      if (cache[i].kern == kern && cache[i].dev == dev) return cache[i].pairs;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(2 * (num_sms() / 2));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int pairs = 0;
  if (cudaOccupancyMaxActiveClusters(&pairs, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    pairs = 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (n_cache < 64) cache[n_cache++] = {kern, dev, pairs};
  return pairs;
}

template <int EPI, int HD, int BN, int ST>
int launch_pair_bn(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, int M, int N, int K,
                   const EpiParams& ep, cudaStream_t stream, const char* name) {
  CKV_REQUIRE(a && b, "%s: null operand", name);
  CKV_REQUIRE(M >= 0 && N > 0 && K > 0, "%s: bad sizes m=%d n=%d k=%d", name, M, N, K);
  CKV_REQUIRE(aligned16(a) && aligned16(b), "%s: operands must be 16-byte aligned", name);
  CKV_REQUIRE(K % 8 == 0 && lda % 8 == 0 && ldb % 8 == 0,
              "%s: k and row strides must be multiples of 8", name);
  CKV_REQUIRE(N % 16 == 0, "%s: n=%d must be a multiple of 16", name, N);
  if (M == 0) return CKV_OK;
  CUtensorMap ma, mb;
  if (int rc = make_map(&ma, a, M, K, lda, BM)) return rc;
  if (int rc = make_map(&mb, b, N, K, ldb, BN / 2)) return rc;
  auto kern = gemm_pair_kernel<EPI, HD, BN, ST>;
  constexpr int smem = PCfg<BN, ST>::SMEM_BYTES;
  if (int rc = set_smem_limit(reinterpret_cast<const void*>(kern), smem)) return rc;
  const int tiles = ceil_div(M, 2 * BM) * ceil_div(N, BN);
  int pairs = resident_pairs(reinterpret_cast<const void*>(kern), smem);
  if (pairs <= 0) pairs = num_sms() / 2;
  pairs = std::max(1, std::min(tiles, pairs));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // dependent launch
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, ma, mb, M, N, K, ep) != cudaSuccess) {
    set_error("%s: launch failed: %s", name, cudaGetErrorString(cudaGetLastError()));
    return CKV_ERR_CUDA;
  }
  CKV_LAUNCH_CHECK(name);
  return CKV_OK;
}

// Makespan of whole tiles, in column units: waves x tile width.
int64_t makespan(int M, int N, int bn) {
  const int tiles = ceil_div(M, BM) * ceil_div(N, bn);
  return int64_t(ceil_div(tiles, num_sms())) * bn;
}
// The same for 256-row pair tiles on the SM pairs.
int64_t makespan_pair(int M, int N, int bn) {
  const int tiles = ceil_div(M, 2 * BM) * ceil_div(N, bn);
  return int64_t(ceil_div(tiles, std::max(1, num_sms() / 2))) * bn;
}

// SwiGLU (interleaved 128-column blocks) and QKV (whole heads) tiles stay 256 wide;
// the plain and residual epilogues take 224 when it finishes sooner.
template <int EPI, int HD>
int launch(const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb, int M, int N, int K,
           const EpiParams& ep, cudaStream_t stream, const char* name) {
  // 256-row tiles on SM pairs when every pair gets two tiles or more (the k-loop then
  // dominates, and the pair's lighter operand traffic pays); a single wave of tiles
  // mostly gains nothing from it (measured at M = 938: o_proj and qkv slower)
  if (int64_t(ceil_div(M, 2 * BM)) * ceil_div(N, 256) >= 2 * int64_t(num_sms() / 2)) {
    if constexpr (EPI == EPI_STORE || EPI == EPI_RESID || EPI == EPI_PARTIAL) {
      const int64_t m256 = makespan_pair(M, N, 256), m224 = makespan_pair(M, N, 224),
                    m208 = makespan_pair(M, N, 208);
      if (m208 < m224 && m208 < m256)
        return launch_pair_bn<EPI, HD, 208, 7>(a, lda, b, ldb, M, N, K, ep, stream, name);
      if (m224 < m256) return launch_pair_bn<EPI, HD, 224, 7>(a, lda, b, ldb, M, N, K, ep, stream, name);
    }
    return launch_pair_bn<EPI, HD, 256, 6>(a, lda, b, ldb, M, N, K, ep, stream, name);
  }
  // the residual GEMM with a long K loop (down_proj) is the exception: 256 x 256 pair
  // tiles, fewer of them than SMs, measured 110 us against 114 us for 128 x 208 tiles on
  // single SMs at M = 938, K = 18944 (same box)
  if constexpr (EPI == EPI_RESID) {
    if (K >= 8192 && M > BM) return launch_pair_bn<EPI, HD, 256, 6>(a, lda, b, ldb, M, N, K, ep, stream, name);
  }
  if constexpr (EPI == EPI_STORE || EPI == EPI_RESID || EPI == EPI_PARTIAL) {
    if (M > 0) {
      const int64_t m256 = makespan(M, N, 256), m224 = makespan(M, N, 224), m208 = makespan(M, N, 208);
      // a long K loop (one tile per SM for a long time) gains from a fifth stage in flight;
      // a short one loses (less L1 left for the epilogue): measured at K = 18944 / 3584
      const bool deep = K >= 8192;
      if (m208 < m224 && m208 < m256)
        return deep ? launch_bn<EPI, HD, 208, 5>(a, lda, b, ldb, M, N, K, ep, stream, name)
                    : launch_bn<EPI, HD, 208, 4>(a, lda, b, ldb, M, N, K, ep, stream, name);
      if (m224 < m256)
        return deep ? launch_bn<EPI, HD, 224, 5>(a, lda, b, ldb, M, N, K, ep, stream, name)
                    : launch_bn<EPI, HD, 224, 4>(a, lda, b, ldb, M, N, K, ep, stream, name);
    }
  }
  return launch_bn<EPI, HD, 256>(a, lda, b, ldb, M, N, K, ep, stream, name);
}

EpiParams zero_params() {
  EpiParams ep;
  memset(&ep, 0, sizeof(ep));
  return ep;
}

}  // namespace
}  // namespace ckv

using namespace ckv;

extern "C" {

int ckv_linear_partial(const uint16_t* x, const uint16_t* w, uint16_t* out, int m, int n, int k,
                       const uint64_t* flags, uint32_t* ticket, int rank, int ranks,
                       ckv_stream_t stream) {
  CKV_REQUIRE(out && flags && ticket && aligned16(out), "ckv_linear_partial: null or unaligned pointer");
  CKV_REQUIRE(ranks >= 1 && ranks <= CKV_MAX_RANKS && rank >= 0 && rank < ranks,
              "ckv_linear_partial: rank %d of %d", rank, ranks);
  if (m <= 0) return CKV_OK;
  EpiParams ep = zero_params();
  ep.out = out;
  ep.ldo = n;
  ep.push_flag = flags;
  ep.push_ticket = ticket;
  ep.push_rank = rank;
  ep.push_ranks = ranks;
  return launch<EPI_PARTIAL, 128>(x, k, w, k, m, n, k, ep, as_stream(stream), "ckv_linear_partial");
}

int ckv_linear(const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* out, int m,
               int n, int k, ckv_stream_t stream) {
  CKV_REQUIRE(out && aligned16(out), "ckv_linear: output must be 16-byte aligned");
  EpiParams ep = zero_params();
  ep.bias = bias;
  ep.out = out;
  ep.ldo = n;
  return launch<EPI_STORE, 128>(x, k, w, k, m, n, k, ep, as_stream(stream), "ckv_linear");
}

int ckv_linear_residual(const uint16_t* x, const uint16_t* w, uint16_t* h, int m, int n, int k,
                        ckv_stream_t stream) {
  CKV_REQUIRE(h && aligned16(h), "ckv_linear_residual: h must be 16-byte aligned");
  EpiParams ep = zero_params();
  ep.out = h;
  ep.ldo = n;
  return launch<EPI_RESID, 128>(x, k, w, k, m, n, k, ep, as_stream(stream),
                                "ckv_linear_residual");
}

int ckv_linear_swiglu(const uint16_t* x, const uint16_t* w_gate_up, uint16_t* out, int m,
                      int inter, int k, ckv_stream_t stream) {
  CKV_REQUIRE(out && aligned16(out), "ckv_linear_swiglu: output must be 16-byte aligned");
  CKV_REQUIRE(inter > 0 && inter % 128 == 0, "ckv_linear_swiglu: inter %% 128 != 0");
  EpiParams ep = zero_params();
  ep.out = out;
  ep.ldo = inter;
  return launch<EPI_SWIGLU, 128>(x, k, w_gate_up, k, m, 2 * inter, k, ep, as_stream(stream),
                                 "ckv_linear_swiglu");
}

int ckv_qkv_rope(const uint16_t* x, const uint16_t* w_qkv, const uint16_t* b_qkv, int m, int k,
                 int col_begin, int col_end, int n_q_heads, int n_kv_heads, int head_dim,
                 const int32_t* positions, const float* rope_table, int rope_max_pos,
                 uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, int n_ctx,
                 uint16_t* k_compact, uint16_t* v_compact, ckv_stream_t stream) {
  CKV_REQUIRE(head_dim == 64 || head_dim == 128, "ckv_qkv_rope: head_dim %d (64 or 128)",
              head_dim);
  CKV_REQUIRE(b_qkv && positions && rope_table, "ckv_qkv_rope: null bias/positions/table");
  const int total = (n_q_heads + 2 * n_kv_heads) * head_dim;
  CKV_REQUIRE(0 <= col_begin && col_begin < col_end && col_end <= total,
              "ckv_qkv_rope: column range [%d,%d) outside [0,%d)", col_begin, col_end, total);
  CKV_REQUIRE(col_begin % head_dim == 0 && col_end % head_dim == 0,
              "ckv_qkv_rope: column range must cover whole heads");
  const bool has_q = col_begin < n_q_heads * head_dim;
  const bool has_kv = col_end > n_q_heads * head_dim;
  CKV_REQUIRE(!has_q || (q_out && aligned16(q_out)), "ckv_qkv_rope: q_out required");
  if (has_kv) {
    const bool cache = k_cache && v_cache;
    const bool compact = k_compact && v_compact;
    CKV_REQUIRE(cache != compact, "ckv_qkv_rope: give either k/v caches or compact k/v buffers");
    CKV_REQUIRE(cache ? (aligned16(k_cache) && aligned16(v_cache) && n_ctx > 0)
                      : (aligned16(k_compact) && aligned16(v_compact)),
                "ckv_qkv_rope: k/v outputs must be 16-byte aligned");
  }
  CKV_REQUIRE(rope_max_pos > 0, "ckv_qkv_rope: empty rope table");
  EpiParams ep = zero_params();
  ep.bias = b_qkv;
  ep.positions = positions;
  ep.rope = reinterpret_cast<const float2*>(rope_table);
  ep.rope_max_pos = rope_max_pos;
  ep.col_begin = col_begin;
  ep.n_q_heads = n_q_heads;
  ep.n_kv_heads = n_kv_heads;
  ep.q_out = q_out;
  ep.k_cache = k_cache;
  ep.v_cache = v_cache;
  ep.n_ctx = n_ctx;
  ep.k_compact = k_compact;
  ep.v_compact = v_compact;
  const uint16_t* wb = w_qkv + int64_t(col_begin) * k;
  const int n = col_end - col_begin;
  if (head_dim == 128)
    return launch<EPI_QKV, 128>(x, k, wb, k, m, n, k, ep, as_stream(stream), "ckv_qkv_rope");
  return launch<EPI_QKV, 64>(x, k, wb, k, m, n, k, ep, as_stream(stream), "ckv_qkv_rope");
}

}  // extern "C"
