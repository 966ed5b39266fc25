// Layer-1 K/V deviation + pooled top-k selection (torch_engine.py:117-153).
//
// One launch, in clusters of kCluster CTAs.  Phase 1 (every CTA, a balanced block of
// active rows each, one warp per row with all of the row's loads in flight):
//   diff = sum_{h,d} fp32(bf16(k - K))^2 + sum fp32(bf16(v - V))^2   (torch_engine.py:118-119)
//   norm = sum fp32(k)^2 + sum fp32(v)^2                             (torch_engine.py:120)
// and, for rows that are eligible unless their chunk escalates (cached, not a sink,
// inside a pooled chunk), a shared-memory histogram of the top 11 bits of the score,
// added into a global histogram in the control block.
// Phase 2 (the last cluster to finish, found with an atomic ticket — no waiting): the
// cluster's CTAs each hold one contiguous slice of the positions (a score key and a
// flag byte per position, in shared memory) and exchange what crosses slices through
// distributed shared memory, between hardware cluster barriers:
//   per-chunk rel = sum diff / sum norm over the chunk span           (torch_engine.py:132)
//     (each CTA sums its slice, the slice sums are added in rank order)
//   keep = ~cached | sink | escalated spans; pool = pooled spans     (torch_engine.py:125-140)
//   budget = min(sum of per-chunk budgets, |pool & ~keep|)          (torch_engine.py:139,142)
//   top-`budget` eligible positions by diff: a three-level radix select (11, 11 and 9
//     bits) on the fp32 bit pattern of diff >= 0, each level's histogram the sum of the
//     slices' (the first level's is phase 1's unless a chunk escalated, an exact
//     position lies in the pool, or there was no phase 1); equal scores: lower
//     position first — the reference's argsort leaves that order undefined,
//     torch_engine.py:144
//   keep_abs = ascending kept positions, sel = index in the active list (146-150),
//     each slice at the offset the lower slices' counts give.
#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(select)

#include <cooperative_groups.h>

#include <mutex>

namespace cg = cooperative_groups;

namespace ckv {
namespace {

// 512 threads: two CTAs fit on an SM (64 registers each), so an 8-CTA cluster packs
// into four SMs and the resident clusters cover every SM
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
static_assert(kWarps <= 32, "one warp scans the warp totals");
constexpr int kCluster = 8;  // CTAs of one cluster; the last cluster runs the selection
// positions of one CTA's slice held in shared memory (9 bytes each: key, flags and
// norm), beside the chunk partials (8 bytes per chunk) and about 17 KiB of static
// shared memory
constexpr int kSmemSlice = 20128;
constexpr int kMaxChunks = 4096;        // chunk table the selection takes
// chunk tables up to this size are copied to shared memory for phase 1's histogram
constexpr int kPhase1Chunks = 1024;
constexpr int kBins = 2048;  // first radix level: score bits [30:20]

// pos_flags input bits
constexpr uint8_t kInCached = 1, kInSink = 2, kInExact = 4;
// working flag bits
constexpr uint8_t kKeep = 1, kExact = 2, kCached = 4, kPool = 8;

// Control block (global, CKV_SELECT_CONTROL_BYTES): ticket counter, then the phase-1
// histogram.  Zero before the first launch; every launch leaves it zero.
struct Control {
  unsigned ticket;
  unsigned pad[63];
  unsigned hist[kBins];
};
static_assert(sizeof(Control) == CKV_SELECT_CONTROL_BYTES, "control block layout");

struct SelectArgs {
  const float* diff;
  const float* norm;
  const uint8_t* pos_flags;
  int n_ctx;
  const int32_t* meta;  // [n_chunks][4] start, length, budget(-1 = not pooled), exact
  int n_chunks;
  int has_thr;
  double thr;
  float* rel;
  int32_t* keep_abs;
  int32_t* sel;
  int32_t* counts;
  uint32_t* keys_scratch;   // [round16(n_ctx)] used when a slice exceeds kSmemSlice
  uint8_t* flags_scratch;   // [round16(n_ctx)]
};

__host__ __device__ constexpr int round16(int n) { return (n + 15) / 16 * 16; }
// positions per CTA slice (a multiple of 16, so every slice starts 64-byte aligned)
__host__ __device__ constexpr int slice_len(int n_ctx) { return round16((n_ctx + kCluster - 1) / kCluster); }
__host__ __device__ constexpr bool slice_in_smem(int n_ctx) { return slice_len(n_ctx) <= kSmemSlice; }
// dynamic shared memory: the slice's keys, flags and norms (when they fit), then the
// chunk partials; phase 1's copy of the chunk table shares the same bytes
__host__ __device__ constexpr int dyn_smem_bytes(int n_ctx, int n_chunks) {
  return (slice_in_smem(n_ctx) ? 9 * slice_len(n_ctx) : 0) + 16 * ((n_chunks + 1) / 2) >
                 16 * (n_chunks < kPhase1Chunks ? n_chunks : kPhase1Chunks)
             ? (slice_in_smem(n_ctx) ? 9 * slice_len(n_ctx) : 0) + 16 * ((n_chunks + 1) / 2)
             : 16 * (n_chunks < kPhase1Chunks ? n_chunks : kPhase1Chunks);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// inclusive scan over the lanes
__device__ __forceinline__ int warp_incl(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Exclusive scan over the kWarps warps of one int per warp (lane 0's value counts);
// returns the warp's base, *total the CTA sum.  All kThreads threads call it.
__device__ int warp_bases(int v, int* total, int* s_w) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) s_w[warp] = v;
  __syncthreads();
  if (warp == 0) {
    const int x = lane < kWarps ? s_w[lane] : 0;
    const int inc = warp_incl(x);
    if (lane < kWarps) s_w[lane] = inc - x;
    if (lane == kWarps - 1) s_w[kWarps] = inc;
  }
  __syncthreads();
  const int base = s_w[warp];
  *total = s_w[kWarps];
  __syncthreads();
  return base;
}

// Ordering key of a score: the bit pattern of a non-negative fp32 value is monotonic in
// it.  -0, negative values and NaN (never produced by sums of squares of finite
// values) rank lowest.
__device__ __forceinline__ uint32_t score_key(float d) {
  const uint32_t u = __float_as_uint(d);
  return ((u & 0x80000000u) || u > 0x7f800000u) ? 0u : u;
}

// Histogram add.  When every active lane of the warp has the same bin (keys that
// cluster, e.g. every token whose fresh K/V equal the cached ones), one lane adds them
// all; otherwise each lane adds its own (keys mostly in distinct bins).
// Warp-uniform call: every lane of the warp must reach it.
__device__ __forceinline__ void hist_add(uint32_t* hist, uint32_t bin, bool on) {
  const unsigned act = __ballot_sync(0xffffffffu, on);
  if (act == 0u) return;
  const int leader = __ffs(act) - 1;
  const uint32_t b0 = __shfl_sync(0xffffffffu, bin, leader);
  if (__ballot_sync(0xffffffffu, on && bin == b0) == act) {
    if (int(threadIdx.x & 31) == leader) atomicAdd(&hist[b0], unsigned(__popc(act)));
  } else if (on) {
    atomicAdd(&hist[bin], 1u);
  }
}

// Bins ranked from the top of this CTA's `hist` (nbins = 2048 or 512, a multiple of
// kThreads): thread t takes the nbins / kThreads bins that follow, from the top, the
// t * nbins / kThreads highest.  Returns the number of keys counted; for
// k' = min(k, that number) > 0, *s_bin and *s_k receive the bin that holds the k'-th
// largest key and the key's rank inside that bin.
__device__ int rank_bins_local(const uint32_t* hist, int nbins, int k, int* s_w, int* s_bin, int* s_k) {
  const int per = nbins / kThreads;  // 4 or 1
  const int top = nbins - 1 - per * int(threadIdx.x);
  int mine = 0;
  for (int i = 0; i < per; ++i) mine += int(hist[top - i]);
  const int inc = warp_incl(mine);
  int tot;
  const int wb = warp_bases(__shfl_sync(0xffffffffu, inc, 31), &tot, s_w);
  int excl = wb + inc - mine;
  const int kk = min(k, tot);
  if (kk > 0 && excl < kk && kk <= excl + mine) {
    for (int i = 0; i < per; ++i) {
      const int c = int(hist[top - i]);
      if (kk - excl <= c) {
        *s_bin = top - i;
        *s_k = kk - excl;
        break;
      }
      excl += c;
    }
  }
  __syncthreads();
  return tot;
}

struct Rank {
  int bin, k, total;
};

// Distributed shared memory: CTA `rank`'s copy of the shared variable at `p`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, unsigned rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ uint4 ld_cluster_v4(const void* p, unsigned rank) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(cluster_addr(p, rank)));
  return v;
}
__device__ __forceinline__ float2 ld_cluster_f2(const void* p, unsigned rank) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(cluster_addr(p, rank)));
  return v;
}
__device__ __forceinline__ int ld_cluster_i32(const void* p, unsigned rank) {
  int v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr(p, rank)));
  return v;
}
// A cluster barrier in two halves: arrive (release) once this CTA's shared values that
// the others read are written, or once its reads of theirs are done; wait (acquire)
// before relying on the others.  Local work between the two hides the barrier.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// The cluster-wide ranking of a level: every CTA sums the kCluster CTAs' copies of `h`
// itself (thread t: bins [nbins - 4t - 4, nbins - 4t), one 16-byte remote read per CTA,
// all in flight at once) and ranks the sums from the top, so no CTA waits for another
// one's answer.  Called by every thread after a cluster barrier that follows the last
// update of any copy; *s_bin and *s_k as in rank_bins_local.
__device__ int rank_bins_merged(const uint32_t* h, int nbins, int k, int* s_w, int* s_bin, int* s_k) {
  const int t = threadIdx.x;
  uint32_t c[4] = {0u, 0u, 0u, 0u};  // highest bin first
  if (4 * t < nbins) {
    const uint32_t* q = h + nbins - 4 * (t + 1);
    uint4 v[kCluster];
#pragma unroll
    for (int r = 0; r < kCluster; ++r) v[r] = ld_cluster_v4(q, unsigned(r));
#pragma unroll
    for (int r = 0; r < kCluster; ++r) {
      c[0] += v[r].w;
      c[1] += v[r].z;
      c[2] += v[r].y;
      c[3] += v[r].x;
    }
  }
  const int mine = int(c[0] + c[1] + c[2] + c[3]);
  const int inc = warp_incl(mine);
  int tot;
  const int wb = warp_bases(__shfl_sync(0xffffffffu, inc, 31), &tot, s_w);
  int excl = wb + inc - mine;
  const int kk = min(k, tot);
  if (kk > 0 && excl < kk && kk <= excl + mine) {
    for (int i = 0; i < 4; ++i) {
      if (kk - excl <= int(c[i])) {
        *s_bin = nbins - 1 - 4 * t - i;
        *s_k = kk - excl;
        break;
      }
      excl += int(c[i]);
    }
  }
  __syncthreads();
  return tot;
}

__device__ __forceinline__ bool eligible(uint32_t f) { return (f & kPool) && !(f & kKeep); }
__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xffu; }

// fl[p - lo] |= bit for p in [s, e) ∩ [lo, hi), by one warp, eight reads in flight per
// lane.  Returns (on every lane) whether a byte that gained the bit had `watch` set and
// not kKeep.
__device__ __forceinline__ bool set_span_bit(uint8_t* fl, int lo, int hi, int s, int e, uint8_t bit,
                                             uint8_t watch) {
  const int lane = threadIdx.x & 31;
  s = max(s, lo) - lo;
  e = min(e, hi) - lo;
  bool seen = false;
  for (int q = s + lane; q < e; q += 8 * 32) {
    uint8_t f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = q + 32 * j < e ? fl[q + 32 * j] : uint8_t(0);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (q + 32 * j < e) {
        fl[q + 32 * j] = f[j] | bit;
        seen |= (f[j] & watch) && !(f[j] & kKeep);
      }
  }
  return __any_sync(0xffffffffu, seen);
}

// Row c of the chunk table: start, length, budget, exact.
__device__ __forceinline__ int4 chunk_row(const int32_t* meta, int c) {
  const int32_t* m = meta + c * CKV_SEL_META_STRIDE;
  return make_int4(m[0], m[1], m[2], m[3]);
}

struct TailShared {
  int w[kWarps + 1];
  int wc[4][kWarps];  // per warp of the final pass: eligible keys above thr, equal to it,
                      // other kept positions, exact positions
  int wp[2][kWarps];  // exclusive prefixes over the warps of wc[1] and wc[3]
  __align__(16) int tot[4];  // this CTA's sums of wc, read by the others
  int base[3];               // eq keys, kept and exact positions of the lower slices
  int n_sel;
  int x5;  // an exact position of this slice lies in the pool
  int budget, bin, k, slow;
  unsigned escmask;
  unsigned esc[kMaxChunks / 32];
};

// One radix level's counts of this CTA's slice into its own `h` (cleared here): eligible
// keys whose bits [31:shift] equal prefix's, binned by the nbits below them.
__device__ __forceinline__ void count_level(uint32_t* h, const uint32_t* keys, const uint8_t* fl, int g_lo,
                                            int g_hi, uint32_t prefix, int shift, int nbits) {
  const int lane = threadIdx.x & 31;
  const int nbins = 1 << nbits;
  for (int i = threadIdx.x; i < nbins; i += kThreads) h[i] = 0u;
  __syncthreads();
  for (int g0 = g_lo; g0 < g_hi; g0 += 32) {
    const int g = g0 + lane;
    uint4 k = make_uint4(0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu);
    uint32_t f = 0u;
    if (g < g_hi) {
      k = *reinterpret_cast<const uint4*>(keys + 4 * g);
      f = *reinterpret_cast<const uint32_t*>(fl + 4 * g);
    }
    const uint32_t kk[4] = {k.x, k.y, k.z, k.w};
    bool any = false;
    bool on[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      on[i] = (kk[i] >> shift) == (prefix >> shift) && eligible(byte_of(f, i));
      any |= on[i];
    }
    if (__any_sync(0xffffffffu, any)) {
#pragma unroll
      for (int i = 0; i < 4; ++i) hist_add(h, (kk[i] >> (shift - nbits)) & uint32_t(nbins - 1), on[i]);
    }
  }
}

// Phase 2: the selection, by the kCluster CTAs of one cluster (kThreads threads each).
// keys/fl: this CTA's slice [rank * S, rank * S + S) of the positions, in shared or
// global memory (16-byte aligned); nrm: the slice's norms staged in shared memory, or
// nullptr (read from global memory); part: n_chunks float2 in shared memory; hist: kBins
// shared counters; phase1_hist: the control block's histogram (nullptr: none usable),
// read by every CTA and cleared by rank 0.
__device__ void select_tail(cg::cluster_group& cluster, const SelectArgs& a, uint32_t* keys, uint8_t* fl,
                            float* nrm, float2* part, uint32_t* hist, unsigned* phase1_hist) {
  __shared__ TailShared t;
  __shared__ __align__(16) uint32_t hist2[kBins];  // the second level's counters
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rank = int(cluster.block_rank());
  const int n = a.n_ctx;
  const int S = slice_len(n);
  const int lo = min(n, rank * S), hi = min(n, lo + S);
  const int nl = hi - lo;            // positions of this slice
  const int nq = (nl + 3) >> 2;      // quads of them

  if (phase1_hist)
    for (int i = tid; i < kBins; i += kThreads) hist[i] = __ldcg(phase1_hist + i);
  if (tid == 0) {
    t.budget = 0;
    t.escmask = 0u;
    t.slow = phase1_hist ? 0 : 1;
    t.x5 = 0;
    if (rank == 0) {  // the counts every CTA adds to (step 8)
      a.counts[1] = 0;
      a.counts[5] = 0;
      a.counts[6] = 0;
    }
  }
  for (int i = tid; i < kMaxChunks / 32; i += kThreads) t.esc[i] = 0u;

  // 1. this slice's raw flags, scores and norms (torch_engine.py:121-122: positions
  // never computed score 0), four positions per lane and four quads per thread in
  // flight, vector loads where the inputs allow
  const bool vec_in = ((reinterpret_cast<uintptr_t>(a.pos_flags + lo) & 3u) == 0) &&
                      ((reinterpret_cast<uintptr_t>(a.diff + lo) & 15u) == 0) &&
                      ((reinterpret_cast<uintptr_t>(a.norm + lo) & 15u) == 0);
  for (int g0 = tid; g0 < nq; g0 += 4 * kThreads) {
    uint32_t f4[4];
    uint4 d4[4];
    float4 n4[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int g = g0 + u * kThreads;
      const int p = lo + 4 * g;
      f4[u] = 0u;
      d4[u] = make_uint4(0u, 0u, 0u, 0u);
      n4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (g < nq) {
        if (vec_in && p + 3 < hi) {
          f4[u] = __ldcg(reinterpret_cast<const unsigned*>(a.pos_flags + p));
          d4[u] = __ldcg(reinterpret_cast<const uint4*>(a.diff + p));
          if (nrm) n4[u] = __ldcg(reinterpret_cast<const float4*>(a.norm + p));
        } else {
          uint32_t* dd = reinterpret_cast<uint32_t*>(&d4[u]);
          float* nn = reinterpret_cast<float*>(&n4[u]);
          for (int i = 0; i < 4 && p + i < hi; ++i) {
            f4[u] |= uint32_t(a.pos_flags[p + i]) << (8 * i);
            dd[i] = __float_as_uint(__ldcg(a.diff + p + i));
            if (nrm) nn[i] = __ldcg(a.norm + p + i);
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int g = g0 + u * kThreads;
      if (g < nq) {
        *reinterpret_cast<uint32_t*>(fl + 4 * g) = f4[u];  // raw pos_flags for now
        *reinterpret_cast<uint4*>(keys + 4 * g) = d4[u];   // raw diff bits for now
        if (nrm) *reinterpret_cast<float4*>(nrm + 4 * g) = n4[u];
      }
    }
  }
  __syncthreads();

  // 2. per chunk, this slice's share of its span: (sum diff, sum norm) over the
  // positions that were computed (torch_engine.py:128-132).  Warp w takes chunks w,
  // w + kWarps, ...; lane j fetches the table row of the warp's j-th chunk, so one
  // round of loads covers 32 chunks per warp.
  for (int c0 = 0; c0 < a.n_chunks; c0 += 32 * kWarps) {
    const int c = c0 + warp + kWarps * lane;
    const int4 m = c < a.n_chunks ? chunk_row(a.meta, c) : make_int4(0, 0, -1, 1);
    const bool span = c < a.n_chunks && !m.w && max(m.x, lo) < min(m.x + m.y, hi);
    if (c < a.n_chunks && !span) part[c] = make_float2(0.f, 0.f);
    unsigned todo = __ballot_sync(0xffffffffu, span);
    while (todo) {
      const int j = __ffs(todo) - 1;
      todo &= todo - 1;
      const int ms = __shfl_sync(0xffffffffu, m.x, j), ml = __shfl_sync(0xffffffffu, m.y, j);
      const int s = max(ms, lo), e = min(ms + ml, hi);
      float sd = 0.f, sn = 0.f;
      for (int q = s + lane; q < e; q += 8 * 32) {
        float dd[8], nn[8];
        bool use[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int p = q + 32 * i;
          use[i] = p < e && !(fl[p - lo] & kInExact);
          dd[i] = use[i] ? __uint_as_float(keys[p - lo]) : 0.f;
          nn[i] = use[i] ? (nrm ? nrm[p - lo] : __ldcg(a.norm + p)) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          sd += dd[i];
          sn += nn[i];
        }
      }
      sd = warp_sum(sd);
      sn = warp_sum(sn);
      if (lane == 0) part[c0 + warp + kWarps * j] = make_float2(sd, sn);
    }
  }
  __syncthreads();  // partials written; the raw values are read
  cluster_arrive();

  // 4. (under the barrier) per-position state: keep = ~cached | sink
  // (torch_engine.py:125), the score key
  for (int g = tid; g < nq; g += kThreads) {
    const uint32_t f4 = *reinterpret_cast<const uint32_t*>(fl + 4 * g);
    const uint4 d4 = *reinterpret_cast<const uint4*>(keys + 4 * g);
    const uint32_t d[4] = {d4.x, d4.y, d4.z, d4.w};
    uint32_t w = 0;
    uint4 k;
    uint32_t* kk = reinterpret_cast<uint32_t*>(&k);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t f = byte_of(f4, i);
      const bool in = 4 * g + i < nl;
      uint32_t b = 0;
      if (in) {
        if (!(f & kInCached) || (f & kInSink)) b |= kKeep;
        if (f & kInExact) b |= kExact;
        if (f & kInCached) b |= kCached;
      }
      w |= b << (8 * i);
      kk[i] = (in && !(f & kInExact)) ? score_key(__uint_as_float(d[i])) : 0u;
    }
    *reinterpret_cast<uint32_t*>(fl + 4 * g) = w;
    *reinterpret_cast<uint4*>(keys + 4 * g) = k;
  }
  cluster_wait();  // every slice's partials are written
  if (phase1_hist && rank == 0)  // every CTA has its copy: clear it for the next launch
    for (int i = tid; i < kBins; i += kThreads) phase1_hist[i] = 0u;

  // 3. rel of every chunk from the slices' partials in rank order; escalation, budget
  // (torch_engine.py:128-140) — the same values in every CTA
  for (int c = tid; c < a.n_chunks; c += kThreads) {
    const int4 m = chunk_row(a.meta, c);
    if (m.w) continue;  // exact
    float2 v[kCluster];
#pragma unroll
    for (int r = 0; r < kCluster; ++r) v[r] = ld_cluster_f2(part + c, unsigned(r));
    float sd = 0.f, sn = 0.f;
#pragma unroll
    for (int r = 0; r < kCluster; ++r) {
      sd += v[r].x;
      sn += v[r].y;
    }
    const float rel = __fdiv_rn(sd, sn);
    const bool esc = a.has_thr && (double(rel) > a.thr);
    if (rank == 0) a.rel[c] = rel;
    if (esc) {
      atomicOr(&t.esc[c >> 5], 1u << (c & 31));
      if (c < 32) atomicOr(&t.escmask, 1u << c);
      t.slow = 1;  // phase 1 counted the span's rows as eligible
    } else if (m.z >= 0) {
      atomicAdd(&t.budget, m.z);
    }
  }
  __syncthreads();

  // 5. escalated spans kept whole (torch_engine.py:133-135), then pool = spans of
  // pooled, non-escalated chunks (136-140); an exact position in the pool was never
  // computed, so phase 1 did not count it
  for (int pass = 0; pass < 2; ++pass) {
    for (int c0 = 0; c0 < a.n_chunks; c0 += 32 * kWarps) {
      const int c = c0 + warp + kWarps * lane;
      const int4 m = c < a.n_chunks ? chunk_row(a.meta, c) : make_int4(0, 0, -1, 1);
      const bool esc = c < a.n_chunks && ((t.esc[c >> 5] >> (c & 31)) & 1u);
      const bool go = c < a.n_chunks && !m.w && max(m.x, lo) < min(m.x + m.y, hi) &&
                      (pass == 0 ? esc : (!esc && m.z >= 0));
      unsigned todo = __ballot_sync(0xffffffffu, go);
      while (todo) {
        const int j = __ffs(todo) - 1;
        todo &= todo - 1;
        const int ms = __shfl_sync(0xffffffffu, m.x, j), ml = __shfl_sync(0xffffffffu, m.y, j);
        if (pass == 0) {
          set_span_bit(fl, lo, hi, ms, ms + ml, kKeep, 0);
        } else if (set_span_bit(fl, lo, hi, ms, ms + ml, kPool, kExact) && lane == 0) {
          t.x5 = 1;
        }
      }
    }
    __syncthreads();
  }
  cluster_arrive();  // every slice's flags are final; x5 of every CTA written

  // 6. radix select of the budget-th largest eligible key (eligible = pool & ~keep,
  // torch_engine.py:142-144): bits [30:20], [19:9], [8:0].  Each CTA counts its slice
  // in warp blocks of quads; the counts of a level are summed over the CTAs.  Under the
  // barrier: phase 1's histogram (the same in every CTA) gives the first level and this
  // slice's second-level counts start, unless escalation already rules phase 1 out.
  const int per_warp = (nq + kThreads - 1) / kThreads * 32;  // quads, a multiple of 32
  const int g_lo = min(nq, warp * per_warp), g_hi = min(nq, g_lo + per_warp);
  int n_elig = 0, bin1 = 0, k1 = 0;
  if (!t.slow) {
    if (tid == 0) {
      t.bin = 0;
      t.k = 0;
    }
    n_elig = rank_bins_local(hist, kBins, t.budget, t.w, &t.bin, &t.k);
    bin1 = t.bin;
    k1 = t.k;
    if (min(t.budget, n_elig) > 0) count_level(hist2, keys, fl, g_lo, g_hi, uint32_t(bin1) << 20, 20, 11);
  }
  cluster_wait();
  int slow = t.slow;
  for (int r = 0; r < kCluster; ++r) slow |= ld_cluster_i32(&t.x5, unsigned(r));
  if (slow) {  // first level from the keys (phase 1's histogram misses positions)
    if (tid == 0) {
      t.bin = 0;
      t.k = 0;
    }
    count_level(hist, keys, fl, g_lo, g_hi, 0u, 31, 11);
    cluster.sync();
    n_elig = rank_bins_merged(hist, kBins, t.budget, t.w, &t.bin, &t.k);
    bin1 = t.bin;
    k1 = t.k;
    if (min(t.budget, n_elig) > 0) count_level(hist2, keys, fl, g_lo, g_hi, uint32_t(bin1) << 20, 20, 11);
  }
  const int budget = min(t.budget, n_elig);
  uint32_t thr = 0x80000000u;  // above every key: nothing selected
  int take_eq = 0;
  if (budget > 0) {  // the same in every CTA
    uint32_t prefix = uint32_t(bin1) << 20;
    // second level: bits [19:9] from hist2 (counted above)
    cluster.sync();
    if (tid == 0) {
      t.bin = 0;
      t.k = 0;
    }
    rank_bins_merged(hist2, kBins, k1, t.w, &t.bin, &t.k);
    prefix |= uint32_t(t.bin) << 9;
    const int k2 = t.k;
    // third level: bits [8:0] into hist, which no CTA reads any more (every CTA passed
    // the barrier above after its last read of the others' hist)
    count_level(hist, keys, fl, g_lo, g_hi, prefix, 9, 9);
    cluster.sync();
    if (tid == 0) {
      t.bin = 0;
      t.k = 0;
    }
    rank_bins_merged(hist, 512, k2, t.w, &t.bin, &t.k);
    thr = prefix | uint32_t(t.bin);
    take_eq = t.k;
  }

  // 7. counts over the slice, per warp: eligible keys above thr and equal to it, other
  // kept positions, exact positions; one exchange gives every CTA the lower slices'
  // totals (torch_engine.py:144-150: the first take_eq equal keys by position are kept)
  {
    int c[4] = {0, 0, 0, 0};
    for (int g = g_lo + lane; g < g_hi; g += 32) {
      const uint4 k = *reinterpret_cast<const uint4*>(keys + 4 * g);
      const uint32_t f = *reinterpret_cast<const uint32_t*>(fl + 4 * g);
      const uint32_t kk[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t b = byte_of(f, i);
        if (eligible(b)) {
          c[0] += kk[i] > thr ? 1 : 0;
          c[1] += kk[i] == thr ? 1 : 0;
        } else {
          c[2] += (b & kKeep) ? 1 : 0;
        }
        c[3] += (b & kExact) ? 1 : 0;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = warp_sum_i(c[j]);
      if (lane == 0) t.wc[j][warp] = s;
    }
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int x = lane < kWarps ? t.wc[j][lane] : 0;
      const int inc = warp_incl(x);
      if (j == 1 && lane < kWarps) t.wp[0][lane] = inc - x;
      if (j == 3 && lane < kWarps) t.wp[1][lane] = inc - x;
      if (lane == 31) t.tot[j] = inc;
    }
  }
  __syncthreads();
  cluster.sync();  // every CTA's totals
  if (warp == 0) {
    int4 v = make_int4(0, 0, 0, 0);
    if (lane < kCluster) {
      const uint4 u = ld_cluster_v4(t.tot, unsigned(lane));
      v = make_int4(int(u.x), int(u.y), int(u.z), int(u.w));
    }
    const int eq_incl = warp_incl(v.y);
    const int eq_before = eq_incl - v.y;  // equal keys of the lower slices
    const int taken = lane < kCluster ? max(0, min(take_eq - eq_before, v.y)) : 0;
    const int kept = v.x + v.z + taken;
    const int kept_incl = warp_incl(kept), ex_incl = warp_incl(v.w);
    if (lane == rank) {
      t.base[0] = eq_before;
      t.base[1] = kept_incl - kept;
      t.base[2] = ex_incl - v.w;
    }
    if (lane == 31) t.n_sel = kept_incl;
  }
  __syncthreads();
  cluster_arrive();  // the others' totals are read; the wait comes before leaving

  // 8. mark and compact: keys above thr, then the first take_eq equal to it by position;
  // kept positions in order (keep_abs) and their index among the computed ones (sel)
  int eq_run = t.base[0] + t.wp[0][warp];
  int ex_run = t.base[2] + t.wp[1][warp];
  int out_run = t.base[1];
  {
    int before = 0;  // kept positions of the lower warps of this CTA
    if (lane < warp) {
      const int eb = t.base[0] + t.wp[0][lane];
      before = t.wc[0][lane] + t.wc[2][lane] + max(0, min(take_eq - eb, t.wc[1][lane]));
    }
    out_run += warp_sum_i(before);
  }
  int c_keep = 0, c_cached = 0, c_bad = 0;  // per lane
  for (int g0 = g_lo; g0 < g_hi; g0 += 32) {
    const int g = g0 + lane;
    uint4 k = make_uint4(0u, 0u, 0u, 0u);
    uint32_t f = 0u;
    if (g < g_hi) {
      k = *reinterpret_cast<const uint4*>(keys + 4 * g);
      f = *reinterpret_cast<const uint32_t*>(fl + 4 * g);
    }
    const uint32_t kk[4] = {k.x, k.y, k.z, k.w};
    int n_eq = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) n_eq += (kk[i] == thr && eligible(byte_of(f, i))) ? 1 : 0;
    const int inc = warp_incl(n_eq);
    int r = eq_run + inc - n_eq;  // equal keys before this quad
    eq_run += __shfl_sync(0xffffffffu, inc, 31);
    uint32_t kept4 = 0u;
    int nk = 0, nx = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t b = byte_of(f, i);
      bool kept;
      if (eligible(b)) {
        kept = kk[i] > thr;
        if (kk[i] == thr) kept = (r++ < take_eq);
      } else {
        kept = (b & kKeep) != 0;
      }
      if (kept) {
        kept4 |= 1u << i;
        ++nk;
        if (b & kCached) ++c_cached;
        if (b & kExact) ++c_bad;
      }
      if (b & kExact) ++nx;
    }
    c_keep += nk;
    const int inc2 = warp_incl(nk | (nx << 16));  // both counts fit 16 bits per step
    int ik = out_run + (inc2 & 0xffff) - nk;
    int ix = ex_run + (inc2 >> 16) - nx;
    const int all = __shfl_sync(0xffffffffu, inc2, 31);
    out_run += all & 0xffff;
    ex_run += all >> 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int p = lo + 4 * g + i;
      if ((kept4 >> i) & 1u) {
        a.keep_abs[ik] = p;
        a.sel[ik] = p - ix;
        ++ik;
      }
      if ((byte_of(f, i) & kExact)) ++ix;
    }
  }
  c_keep = warp_sum_i(c_keep);
  c_cached = warp_sum_i(c_cached);
  c_bad = warp_sum_i(c_bad);
  if (lane == 0) {
    if (c_cached) atomicAdd(&a.counts[1], c_cached);
    if (c_keep - c_cached) atomicAdd(&a.counts[6], c_keep - c_cached);
    if (c_bad) {
      atomicOr(&a.counts[5], int(CKV_DEV_ERR_SELECT_UNCOMPUTED));
      atomicOr(&g_err_word, CKV_DEV_ERR_SELECT_UNCOMPUTED);
    }
  }
  if (rank == 0 && tid == 0) {
    a.counts[0] = t.n_sel;
    a.counts[2] = budget;
    a.counts[3] = n_elig;
    a.counts[4] = int(t.escmask);
    a.counts[7] = 0;
  }
  cluster_wait();  // no CTA leaves while another may still read its shared memory
}

// Phase 1 for one active row i (one warp): diff[p], norm[p] for p = active[i].
// Returns p (on every lane; -1 if the position is out of range) and *d_out = diff[p].
__device__ __forceinline__ int deviation_row(
    int64_t i, const uint16_t* __restrict__ k_fresh, const uint16_t* __restrict__ v_fresh,
    int64_t fstride, const uint16_t* __restrict__ k_base, const uint16_t* __restrict__ v_base,
    const int32_t* __restrict__ active, int H, int D, const uint8_t* __restrict__ pos_flags,
    int n_ctx, float* diff, float* norm, float* d_out) {
  const int lane = threadIdx.x & 31;
  const int p = active[i];
  if (p < 0 || p >= n_ctx) {
    if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
    return -1;
  }
  // the reference compares against a zero-initialised cache (torch_engine.py:97) that
  // only moved chunks fill, so a position no chunk covers compares against zeros
  const bool cached = (pos_flags[p] & kInCached) != 0;
  const int vecs = (H * D) / 8;
  float dk = 0.f, dv = 0.f, nk = 0.f, nv = 0.f;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  // two 16-byte vectors of each of the four rows per lane and step: the whole
  // 4 x 1 KiB of a 7B row (H * D = 512) is in flight at once
  for (int v0 = lane; v0 < vecs; v0 += 64) {
    uint4 kf[2], vf[2], kb[2], vb[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int v = v0 + 32 * u;
      kf[u] = vf[u] = kb[u] = vb[u] = zero;
      if (v < vecs) {
        const int e0 = v * 8, h = e0 / D, d = e0 - h * D;
        kf[u] = *reinterpret_cast<const uint4*>(k_fresh + i * fstride + e0);
        vf[u] = *reinterpret_cast<const uint4*>(v_fresh + i * fstride + e0);
        if (cached) {
          const int64_t boff = (int64_t(h) * n_ctx + p) * D + d;
          kb[u] = *reinterpret_cast<const uint4*>(k_base + boff);
          vb[u] = *reinterpret_cast<const uint4*>(v_base + boff);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint32_t* pkf = reinterpret_cast<const uint32_t*>(&kf[u]);
      const uint32_t* pvf = reinterpret_cast<const uint32_t*>(&vf[u]);
      const uint32_t* pkb = reinterpret_cast<const uint32_t*>(&kb[u]);
      const uint32_t* pvb = reinterpret_cast<const uint32_t*>(&vb[u]);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float kf2[2] = {lo_bf(pkf[w]), hi_bf(pkf[w])};
        const float vf2[2] = {lo_bf(pvf[w]), hi_bf(pvf[w])};
        const float kb2[2] = {lo_bf(pkb[w]), hi_bf(pkb[w])};
        const float vb2[2] = {lo_bf(pvb[w]), hi_bf(pvb[w])};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float ek = bf16_round(__fsub_rn(kf2[e], kb2[e]));
          const float ev = bf16_round(__fsub_rn(vf2[e], vb2[e]));
          dk = __fadd_rn(dk, __fmul_rn(ek, ek));
          dv = __fadd_rn(dv, __fmul_rn(ev, ev));
          nk = __fadd_rn(nk, __fmul_rn(kf2[e], kf2[e]));
          nv = __fadd_rn(nv, __fmul_rn(vf2[e], vf2[e]));
        }
      }
    }
  }
  dk = warp_sum(dk);
  dv = warp_sum(dv);
  nk = warp_sum(nk);
  nv = warp_sum(nv);
  const float d = dk + dv;
  if (lane == 0) {
    diff[p] = d;
    norm[p] = nk + nv;
  }
  *d_out = d;
  return p;
}

struct RowArgs {
  const uint16_t* k_fresh;
  const uint16_t* v_fresh;
  int64_t fstride;
  const uint16_t* k_base;
  const uint16_t* v_base;
  const int32_t* active;
  int n_act;
  int H, D;
  const uint8_t* pos_flags;
  int n_ctx;
  float* diff;
  float* norm;
};

// This CTA's rows: a contiguous block of n_act / gridDim.x (+1) rows, a warp per row.
// With `hist` (and the chunk table `tab` of n_tab chunks in shared memory), rows that
// are eligible unless their chunk escalates add their score's top bits to it.
__device__ __forceinline__ void deviation_rows(const RowArgs& r, uint32_t* hist, const int4* tab,
                                               int n_tab) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = int64_t(blockIdx.x) * r.n_act / gridDim.x;
  const int64_t r1 = int64_t(blockIdx.x + 1) * r.n_act / gridDim.x;
  for (int64_t i = r0 + warp; i < r1; i += kWarps) {
    float d;
    const int p = deviation_row(i, r.k_fresh, r.v_fresh, r.fstride, r.k_base, r.v_base, r.active,
                                r.H, r.D, r.pos_flags, r.n_ctx, r.diff, r.norm, &d);
    if (hist == nullptr || p < 0) continue;
    const uint8_t f = r.pos_flags[p];
    if (!(f & kInCached) || (f & (kInSink | kInExact))) continue;
    bool pooled = false;  // inside any chunk with a budget (torch_engine.py:136-140)
    for (int c0 = 0; c0 < n_tab && !pooled; c0 += 32) {
      bool in = false;
      if (c0 + lane < n_tab) {
        const int4 t = tab[c0 + lane];  // start, length, budget, exact
        in = !t.w && t.z >= 0 && p >= t.x && p < t.x + t.y;
      }
      pooled = __any_sync(0xffffffffu, in);
    }
    if (pooled && lane == 0) atomicAdd(&hist[score_key(d) >> 20], 1u);
  }
}

__global__ void __launch_bounds__(kThreads) deviation_scores_kernel(RowArgs r) {
  deviation_rows(r, nullptr, nullptr, 0);
}

// The tail's per-CTA arrays: keys, flags and norms of this CTA's slice (shared memory;
// keys and flags in the caller's scratch and norms read in place when the slice is too
// long), then the chunk partials.
struct TailArrays {
  uint32_t* keys;
  uint8_t* fl;
  float* nrm;
  float2* part;
};
__device__ __forceinline__ TailArrays tail_arrays(const SelectArgs& sa, unsigned char* dyn, int rank) {
  const int S = slice_len(sa.n_ctx);
  TailArrays t;
  if (slice_in_smem(sa.n_ctx)) {
    t.keys = reinterpret_cast<uint32_t*>(dyn);
    t.fl = dyn + 4 * size_t(S);
    t.nrm = reinterpret_cast<float*>(dyn + 5 * size_t(S));
    t.part = reinterpret_cast<float2*>(dyn + 9 * size_t(S));
  } else {
    t.keys = sa.keys_scratch + size_t(rank) * S;
    t.fl = sa.flags_scratch + size_t(rank) * S;
    t.nrm = nullptr;
    t.part = reinterpret_cast<float2*>(dyn);
  }
  return t;
}

// Launched in clusters of kCluster CTAs (grid a multiple of kCluster).
__global__ void __launch_bounds__(kThreads) deviation_select_kernel(RowArgs r, Control* ctl,
                                                                     SelectArgs sa) {
  extern __shared__ __align__(16) unsigned char dyn_smem[];
  __shared__ __align__(16) uint32_t hist[kBins];
  __shared__ int s_last;
  cg::cluster_group cluster = cg::this_cluster();
  // phase 1: rows, with the first radix level's histogram when the chunk table fits
  const bool with_hist = sa.n_chunks <= kPhase1Chunks;
  int4* tab = reinterpret_cast<int4*>(dyn_smem);
  if (with_hist) {
    for (int i = threadIdx.x; i < kBins; i += kThreads) hist[i] = 0u;
    for (int c = threadIdx.x; c < sa.n_chunks; c += kThreads)
      tab[c] = make_int4(sa.meta[4 * c], sa.meta[4 * c + 1], sa.meta[4 * c + 2], sa.meta[4 * c + 3]);
    __syncthreads();
  }
  deviation_rows(r, with_hist ? hist : nullptr, tab, with_hist ? sa.n_chunks : 0);
  __syncthreads();
  if (with_hist)
    for (int i = threadIdx.x; i < kBins; i += kThreads)
      if (hist[i]) atomicAdd(&ctl->hist[i], hist[i]);
  __threadfence();
  cluster.sync();  // the cluster's rows and histogram shares are all written
  const int rank = int(cluster.block_rank());
  if (rank == 0 && threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&ctl->ticket, 1u);
    const int last = (prev == gridDim.x / kCluster - 1) ? 1 : 0;
    for (int q = 0; q < kCluster; ++q) *cluster.map_shared_rank(&s_last, q) = last;
  }
  cluster.sync();
  if (!s_last) return;  // every CTA of the cluster leaves together
  __threadfence();
  const TailArrays ta = tail_arrays(sa, dyn_smem, rank);
  select_tail(cluster, sa, ta.keys, ta.fl, ta.nrm, ta.part, hist, with_hist ? ctl->hist : nullptr);
  if (rank == 0 && threadIdx.x == 0) ctl->ticket = 0u;  // ready for the next launch
}

// One cluster of kCluster CTAs.
__global__ void __launch_bounds__(kThreads) select_only_kernel(SelectArgs sa) {
  extern __shared__ __align__(16) unsigned char dyn_smem[];
  __shared__ __align__(16) uint32_t hist[kBins];
  cg::cluster_group cluster = cg::this_cluster();
  const TailArrays ta = tail_arrays(sa, dyn_smem, int(cluster.block_rank()));
  select_tail(cluster, sa, ta.keys, ta.fl, ta.nrm, ta.part, hist, nullptr);
}

int check_select(const uint8_t* pos_flags, int n_ctx, const int32_t* meta, int n_chunks,
                 float* rel, int32_t* keep_abs, int32_t* sel, int32_t* counts, uint8_t* scratch) {
  CKV_REQUIRE(pos_flags && rel && keep_abs && sel && counts && scratch,
              "selection: null pointer");
  CKV_REQUIRE(n_chunks == 0 || meta, "selection: null chunk table");
  CKV_REQUIRE(n_ctx > 0 && n_chunks >= 0, "selection: bad sizes");
  CKV_REQUIRE(n_chunks <= kMaxChunks, "selection: %d chunks (at most %d)", n_chunks, kMaxChunks);
  CKV_REQUIRE((reinterpret_cast<uintptr_t>(scratch) & 15u) == 0,
              "selection: scratch must be 16-byte aligned");
  return CKV_OK;
}

SelectArgs make_select_args(const float* diff, const float* norm, const uint8_t* pos_flags,
                            int n_ctx, const int32_t* meta, int n_chunks, int has_thr, double thr,
                            float* rel, int32_t* keep_abs, int32_t* sel, int32_t* counts,
                            uint8_t* scratch) {
  return SelectArgs{diff, norm, pos_flags, n_ctx, meta, n_chunks, has_thr, thr, rel, keep_abs,
                    sel, counts, reinterpret_cast<uint32_t*>(scratch),
                    scratch + 4 * size_t(round16(n_ctx))};
}

cudaLaunchConfig_t cluster_config(int grid, int dyn, cudaStream_t st, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Clusters of the fused kernel that are resident at once for a dynamic shared memory
// size (queried once per device and size); 0 if the query fails.
int resident_clusters(int dyn) {
  struct Entry {
    int dev, dyn, clusters;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int n_cache = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n_cache; ++i)
      if (cache[i].dev == dev && cache[i].dyn == dyn) return cache[i].clusters;
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cluster_config(kCluster * num_sms(), dyn, nullptr, attr);
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, deviation_select_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    clusters = 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (n_cache < 64) cache[n_cache++] = {dev, dyn, clusters};
  return clusters;
}

// Phase-1 grid without clusters (scores only): every resident CTA of the device (queried
// once per device), so every SM gets the same number of rows; at most one CTA per row.
int rows_grid(int n_act) {
  static std::mutex mu;
  static int per_sm[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int blocks = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64) blocks = per_sm[dev];
  }
  if (blocks <= 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, deviation_scores_kernel, kThreads, 0) !=
            cudaSuccess ||
        blocks <= 0) {
      cudaGetLastError();
      blocks = 2;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64) per_sm[dev] = blocks;
  }
  return std::max(1, std::min(n_act, blocks * num_sms()));
}

// Fused grid: as many whole clusters as are resident at once (so every CTA starts at
// once and every SM gets the same number of rows), at most one CTA per row, at least
// one cluster.
int fused_grid(int n_act, int dyn) {
  int clusters = resident_clusters(dyn);
  if (clusters <= 0) clusters = num_sms() / kCluster;
  clusters = std::min(clusters, std::max(1, n_act / kCluster));
  return kCluster * std::max(1, clusters);
}

int launch_fused(const RowArgs& r, void* control, const SelectArgs& sa, cudaStream_t st,
                 const char* name) {
  const int dyn = dyn_smem_bytes(sa.n_ctx, sa.n_chunks);
  if (int rc = set_smem_limit(reinterpret_cast<const void*>(deviation_select_kernel),
                              dyn_smem_bytes(kCluster * kSmemSlice, kMaxChunks)))
    return rc;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = cluster_config(fused_grid(r.n_act, dyn), dyn, st, attr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, deviation_select_kernel, r, static_cast<Control*>(control), sa);
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", name, cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  CKV_LAUNCH_CHECK(name);
  return CKV_OK;
}

}  // namespace
}  // namespace ckv

using namespace ckv;

extern "C" {

int ckv_deviation_select(const uint16_t* k_fresh, const uint16_t* v_fresh,
                         int64_t fresh_row_stride, const uint16_t* k_base,
                         const uint16_t* v_base, const int32_t* active, int n_act,
                         const uint8_t* pos_flags, int n_ctx, const int32_t* sel_meta,
                         int n_chunks, int has_threshold, double escalate_threshold,
                         int n_kv_heads, int head_dim, float* diff, float* norm, float* rel,
                         int32_t* keep_abs, int32_t* sel, int32_t* counts, uint8_t* scratch,
                         void* control, ckv_stream_t stream) {
  if (int rc = check_select(pos_flags, n_ctx, sel_meta, n_chunks, rel, keep_abs, sel, counts,
                            scratch))
    return rc;
  CKV_REQUIRE(k_fresh && v_fresh && k_base && v_base && active && diff && norm && control,
              "ckv_deviation_select: null pointer");
  CKV_REQUIRE(aligned16(k_fresh) && aligned16(v_fresh) && aligned16(k_base) && aligned16(v_base) &&
                  aligned16(control),
              "ckv_deviation_select: K/V and the control block must be 16-byte aligned");
  CKV_REQUIRE(head_dim % 8 == 0 && fresh_row_stride % 8 == 0 && n_kv_heads > 0,
              "ckv_deviation_select: head_dim and row stride must be multiples of 8");
  CKV_REQUIRE(n_act > 0 && n_act <= n_ctx, "ckv_deviation_select: n_act %d out of range", n_act);
  const RowArgs r{k_fresh, v_fresh, fresh_row_stride, k_base, v_base, active, n_act,
                  n_kv_heads, head_dim, pos_flags, n_ctx, diff, norm};
  const SelectArgs sa = make_select_args(diff, norm, pos_flags, n_ctx, sel_meta, n_chunks,
                                         has_threshold, escalate_threshold, rel, keep_abs, sel,
                                         counts, scratch);
  return launch_fused(r, control, sa, as_stream(stream), "ckv_deviation_select");
}

int ckv_deviation_scores(const uint16_t* k_fresh, const uint16_t* v_fresh,
                         int64_t fresh_row_stride, const uint16_t* k_base, const uint16_t* v_base,
                         const int32_t* active, int n_act, const uint8_t* pos_flags, int n_ctx,
                         int n_kv_heads, int head_dim, float* diff, float* norm,
                         ckv_stream_t stream) {
  CKV_REQUIRE(k_fresh && v_fresh && k_base && v_base && active && pos_flags && diff && norm,
              "ckv_deviation_scores: null pointer");
  CKV_REQUIRE(aligned16(k_fresh) && aligned16(v_fresh) && aligned16(k_base) && aligned16(v_base),
              "ckv_deviation_scores: K/V must be 16-byte aligned");
  CKV_REQUIRE(head_dim % 8 == 0 && fresh_row_stride % 8 == 0 && n_kv_heads > 0,
              "ckv_deviation_scores: head_dim and row stride must be multiples of 8");
  CKV_REQUIRE(n_ctx > 0 && n_act >= 0 && n_act <= n_ctx, "ckv_deviation_scores: n_act %d out of range",
              n_act);
  if (n_act == 0) return CKV_OK;
  const RowArgs r{k_fresh, v_fresh, fresh_row_stride, k_base, v_base, active, n_act,
                  n_kv_heads, head_dim, pos_flags, n_ctx, diff, norm};
  deviation_scores_kernel<<<rows_grid(n_act), kThreads, 0, as_stream(stream)>>>(r);
  CKV_LAUNCH_CHECK("ckv_deviation_scores");
  return CKV_OK;
}

int ckv_select_from_scores(const float* diff, const float* norm, const uint8_t* pos_flags,
                           int n_ctx, const int32_t* sel_meta, int n_chunks, int has_threshold,
                           double escalate_threshold, float* rel, int32_t* keep_abs,
                           int32_t* sel, int32_t* counts, uint8_t* scratch, ckv_stream_t stream) {
  if (int rc = check_select(pos_flags, n_ctx, sel_meta, n_chunks, rel, keep_abs, sel, counts,
                            scratch))
    return rc;
  CKV_REQUIRE(diff && norm, "ckv_select_from_scores: null scores");
  const SelectArgs sa = make_select_args(diff, norm, pos_flags, n_ctx, sel_meta, n_chunks,
                                         has_threshold, escalate_threshold, rel, keep_abs, sel,
                                         counts, scratch);
  if (int rc = set_smem_limit(reinterpret_cast<const void*>(select_only_kernel),
                              dyn_smem_bytes(kCluster * kSmemSlice, kMaxChunks)))
    return rc;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = cluster_config(kCluster, dyn_smem_bytes(n_ctx, n_chunks), as_stream(stream), attr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, select_only_kernel, sa);
  if (e != cudaSuccess) {
    set_error("ckv_select_from_scores: launch failed: %s", cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  CKV_LAUNCH_CHECK("ckv_select_from_scores");
  return CKV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of ckv_deviation_select.
//
// Some callers cannot hand this library any memory beyond the tensors they
// already own: a serving loop whose device memory is entirely carved up by its
// own arena or caching allocator (a cudaMalloc there would synchronise the GPU
// or break its memory accounting), or a plain C/FFI host that has the input and
// output buffers but no allocator to make the selection's scratch and control
// block with.  For them both live here, in one file-scope device array that
// every GPU which loads the library keeps until the process exits:
//   bytes [0, CKV_SELECT_CONTROL_BYTES)  the control block (ticket counter and the
//                                        phase-1 histogram)
//   then 5 * CKV_NOALLOC_MAX_CTX bytes   the selection's per-position keys and
//                                        flags (phase 2 uses them only when n_ctx
//                                        exceeds what it keeps in shared memory)
// Its device address is looked up once per device (cudaGetSymbolAddress, on the
// first call made while that device is current).  Every call shares the array:
// the control block is cleared with an async memset on the caller's stream
// before each launch and the keys and flags are rewritten in full, but two calls
// that overlap on the GPU (different streams, no ordering between them) race on it.
#include <atomic>

namespace ckv {
namespace {

static __device__ __align__(256) unsigned char
    g_noalloc_scratch[CKV_SELECT_CONTROL_BYTES + 5 * CKV_NOALLOC_MAX_CTX];

constexpr int kNoAllocMaxDevices = 64;

// Device address of g_noalloc_scratch on the current device (looked up once per
// device).  Two host threads making their first call on one device at the same time
// both look the address up and store the same value; the entries are atomics, so
// that is not a data race.
int noalloc_scratch(unsigned char** out) {
  static std::atomic<unsigned char*> addr[kNoAllocMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    set_error("ckv_deviation_select_noalloc: no usable current device (%s)", cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  unsigned char* a = addr[dev].load(std::memory_order_relaxed);
  if (a == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("ckv_deviation_select_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return CKV_ERR_CUDA;
    }
    a = static_cast<unsigned char*>(p);
    addr[dev].store(a, std::memory_order_relaxed);
  }
  *out = a;
  return CKV_OK;
}

}  // namespace
}  // namespace ckv

extern "C" int ckv_deviation_select_noalloc(
    const uint16_t* k_fresh, const uint16_t* v_fresh, int64_t fresh_row_stride,
    const uint16_t* k_base, const uint16_t* v_base, const int32_t* active, int n_act,
    const uint8_t* pos_flags, int n_ctx, const int32_t* sel_meta, int n_chunks, int has_threshold,
    double escalate_threshold, int n_kv_heads, int head_dim, float* diff, float* norm, float* rel,
    int32_t* keep_abs, int32_t* sel, int32_t* counts, ckv_stream_t stream) {
  CKV_REQUIRE(n_ctx > 0 && n_ctx <= CKV_NOALLOC_MAX_CTX,
              "ckv_deviation_select_noalloc: n_ctx %d outside 1..%d (the size of its built-in "
              "scratch); use ckv_deviation_select with caller-provided scratch",
              n_ctx, CKV_NOALLOC_MAX_CTX);
  unsigned char* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  unsigned char* control = scratch;
  uint8_t* select_scratch = scratch + CKV_SELECT_CONTROL_BYTES;
  if (int rc = check_select(pos_flags, n_ctx, sel_meta, n_chunks, rel, keep_abs, sel, counts,
                            select_scratch))
    return rc;
  CKV_REQUIRE(k_fresh && v_fresh && k_base && v_base && active && diff && norm,
              "ckv_deviation_select_noalloc: null pointer");
  CKV_REQUIRE(aligned16(k_fresh) && aligned16(v_fresh) && aligned16(k_base) && aligned16(v_base),
              "ckv_deviation_select_noalloc: K/V must be 16-byte aligned");
  CKV_REQUIRE(head_dim % 8 == 0 && fresh_row_stride % 8 == 0 && n_kv_heads > 0,
              "ckv_deviation_select_noalloc: head_dim and row stride must be multiples of 8");
  CKV_REQUIRE(n_act > 0 && n_act <= n_ctx, "ckv_deviation_select_noalloc: n_act %d out of range",
              n_act);
  // the control block must start at zero; a memset is a copy, not an allocation
  cudaError_t e = cudaMemsetAsync(control, 0, CKV_SELECT_CONTROL_BYTES, as_stream(stream));
  if (e != cudaSuccess) {
    set_error("ckv_deviation_select_noalloc: clearing the control block failed: %s",
              cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  const RowArgs r{k_fresh, v_fresh, fresh_row_stride, k_base, v_base, active, n_act,
                  n_kv_heads, head_dim, pos_flags, n_ctx, diff, norm};
  const SelectArgs sa = make_select_args(diff, norm, pos_flags, n_ctx, sel_meta, n_chunks,
                                         has_threshold, escalate_threshold, rel, keep_abs, sel,
                                         counts, select_scratch);
  return launch_fused(r, control, sa, as_stream(stream), "ckv_deviation_select_noalloc");
}
