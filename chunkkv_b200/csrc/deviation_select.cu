// Layer-1 K/V deviation + pooled top-k selection (torch_engine.py:117-153).
//
// One launch.  Phase 1 (every CTA, a balanced block of active rows each, one
// warp per row with all of the row's loads in flight):
//   diff = sum_{h,d} fp32(bf16(k - K))^2 + sum fp32(bf16(v - V))^2   (torch_engine.py:118-119)
//   norm = sum fp32(k)^2 + sum fp32(v)^2                             (torch_engine.py:120)
// Phase 2 (the last CTA to finish, found with an atomic ticket — no waiting):
//   per-chunk rel = sum diff / sum norm over the chunk span           (torch_engine.py:132)
//   keep = ~cached | sink | escalated spans; pool = pooled spans     (torch_engine.py:125-140)
//   budget = min(sum of per-chunk budgets, |pool & ~keep|)          (torch_engine.py:139,142)
//   top-`budget` eligible positions by diff: a three-level radix select
//   (11, 11 and 9 bits) on the fp32 bit pattern of diff >= 0, with
//   warp-aggregated shared-memory histograms; equal scores: lower position
//   first — the reference's argsort leaves that order undefined,
//   torch_engine.py:144
//   keep_abs = ascending kept positions, sel = index in the active list (146-150).
// Phase 2 keeps one 4-byte score key and one flag byte per position in shared
// memory when n_ctx <= kSmemPositions, otherwise in the caller's scratch.
#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(select)

namespace ckv {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
// positions whose keys and flags phase 2 holds in shared memory (5 bytes each)
constexpr int kSmemPositions = 20480;
constexpr uint32_t kNotEligible = 0xffffffffu;  // key of a position outside the pool

// pos_flags input bits
constexpr uint8_t kInCached = 1, kInSink = 2, kInExact = 4;
// working flag bits
constexpr uint8_t kKeep = 1, kExact = 2, kCached = 4, kKept = 0x80;

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
  uint32_t* keys_scratch;   // [n_ctx] used when n_ctx > kSmemPositions
  uint8_t* flags_scratch;   // [n_ctx]
};

__host__ __device__ constexpr int dyn_smem_bytes(int n_ctx) {
  return n_ctx <= kSmemPositions ? int((5 * size_t(n_ctx) + 15) / 16 * 16) : 0;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int4 add4(int4 a, int4 b) {
  return make_int4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ int4 sub4(int4 a, int4 b) {
  return make_int4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w);
}
__device__ __forceinline__ int4 shfl_up4(int4 v, int o) {
  return make_int4(__shfl_up_sync(0xffffffffu, v.x, o), __shfl_up_sync(0xffffffffu, v.y, o),
                   __shfl_up_sync(0xffffffffu, v.z, o), __shfl_up_sync(0xffffffffu, v.w, o));
}

// Block-wide exclusive scan of four ints in thread order (all kThreads threads call it);
// *total receives the block sums.
__device__ int4 block_scan4(int4 v, int4* total, int4* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int4 inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int4 t = shfl_up4(inc, o);
    if (lane >= o) inc = add4(inc, t);
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int4 w = s_warp[lane];  // kWarps == 32
    int4 wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int4 t = shfl_up4(wi, o);
      if (lane >= o) wi = add4(wi, t);
    }
    s_warp[lane] = sub4(wi, w);
    if (lane == 31) s_warp[kWarps] = wi;
  }
  __syncthreads();
  const int4 r = add4(s_warp[warp], sub4(inc, v));
  *total = s_warp[kWarps];
  __syncthreads();  // s_warp reusable after return
  return r;
}

// Ordering key of a score: the bit pattern of a non-negative fp32 value is monotonic in
// it.  -0, negative values and NaN (never produced by sums of squares of finite
// values) rank lowest.
__device__ __forceinline__ uint32_t score_key(float d) {
  const uint32_t u = __float_as_uint(d);
  return ((u & 0x80000000u) || u > 0x7f800000u) ? 0u : u;
}

// Histogram add with one shared-memory atomic per distinct bin in the warp (many
// positions share a bin, e.g. every token whose fresh K/V equal the cached ones).
// Warp-uniform call: every lane of the warp must reach it.
__device__ __forceinline__ void hist_add(uint32_t* hist, uint32_t bin, bool on) {
  const unsigned act = __ballot_sync(0xffffffffu, on);
  if (on) {
    const unsigned peers = __match_any_sync(act, bin);
    if (int(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], unsigned(__popc(peers)));
  }
}

// Bins of `hist` (nbins = 2048 or 512) ranked from the top.  Returns the number of
// keys counted; for k' = min(k, that number) > 0, *s_bin and *s_k receive the bin that
// holds the k'-th largest key and the key's rank inside that bin.
__device__ int rank_bins(const uint32_t* hist, int nbins, int k, int4* s_warp, int* s_bin,
                         int* s_k) {
  const int b0 = nbins - 1 - 2 * int(threadIdx.x), b1 = b0 - 1;
  const int c0 = b0 >= 0 ? int(hist[b0]) : 0, c1 = b1 >= 0 ? int(hist[b1]) : 0;
  int4 tot;
  const int excl = block_scan4(make_int4(c0 + c1, 0, 0, 0), &tot, s_warp).x;
  const int kk = min(k, tot.x);
  if (kk > 0 && excl < kk && kk <= excl + c0 + c1) {
    if (kk - excl <= c0) {
      *s_bin = b0;
      *s_k = kk - excl;
    } else {
      *s_bin = b1;
      *s_k = kk - excl - c0;
    }
  }
  __syncthreads();
  return tot.x;
}

// Phase 2: the selection, run by one CTA of kThreads threads.  keys/fl: [n_ctx] each,
// in shared or global memory.
__device__ void select_tail(const SelectArgs& a, uint32_t* keys, uint8_t* fl) {
  __shared__ uint32_t hist[2048];
  __shared__ int4 s_warp[kWarps + 1];
  __shared__ int s_budget, s_bin, s_k;
  __shared__ unsigned s_escmask;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = a.n_ctx;

  // 1. per-position state: keep = ~cached | sink (torch_engine.py:125)
  for (int p = tid; p < n; p += kThreads) {
    const uint8_t f = a.pos_flags[p];
    uint8_t w = 0;
    if (!(f & kInCached) || (f & kInSink)) w |= kKeep;
    if (f & kInExact) w |= kExact;
    if (f & kInCached) w |= kCached;
    fl[p] = w;
    keys[p] = kNotEligible;
  }
  if (tid == 0) {
    s_budget = 0;
    s_escmask = 0u;
  }
  __syncthreads();

  // 2. per chunk: rel over its span (positions never computed count as 0, as in the
  // reference's zero-initialised buffers), escalation keeps the span whole, the
  // budgets of pooled chunks add up (torch_engine.py:128-140)
  for (int c = warp; c < a.n_chunks; c += kWarps) {
    const int32_t* m = a.meta + c * CKV_SEL_META_STRIDE;
    if (m[3]) continue;  // exact
    const int s = max(m[0], 0), e = min(m[0] + m[1], n);
    float sd = 0.f, sn = 0.f;
    for (int p = s + lane; p < e; p += 32) {
      if (fl[p] & kExact) continue;
      sd += __ldcg(a.diff + p);
      sn += __ldcg(a.norm + p);
    }
    sd = warp_sum(sd);
    sn = warp_sum(sn);
    const float rel = __fdiv_rn(sd, sn);
    const bool esc = a.has_thr && (double(rel) > a.thr);
    if (lane == 0) {
      a.rel[c] = rel;
      if (esc && c < 32) atomicOr(&s_escmask, 1u << c);
      if (!esc && m[2] >= 0) atomicAdd(&s_budget, m[2]);
    }
    // overlapping escalated spans set the same bit of a byte no other step changes now
    if (esc)
      for (int p = s + lane; p < e; p += 32) fl[p] |= kKeep;
  }
  __syncthreads();

  // 3. eligible = pool & ~keep gets its score key (torch_engine.py:142-144)
  for (int c = warp; c < a.n_chunks; c += kWarps) {
    const int32_t* m = a.meta + c * CKV_SEL_META_STRIDE;
    if (m[3] || m[2] < 0) continue;
    if (a.has_thr && double(a.rel[c]) > a.thr) continue;  // escalated
    const int s = max(m[0], 0), e = min(m[0] + m[1], n);
    for (int p = s + lane; p < e; p += 32) {
      const uint8_t f = fl[p];
      if (!(f & kKeep)) keys[p] = score_key((f & kExact) ? 0.f : __ldcg(a.diff + p));
    }
  }
  __syncthreads();

  // 4. radix select of the budget-th largest key: bits [30:20], [19:9], [8:0]
  for (int i = tid; i < 2048; i += kThreads) hist[i] = 0u;
  __syncthreads();
  for (int base = warp * 32; base < n; base += kThreads) {
    const int p = base + lane;
    const uint32_t key = p < n ? keys[p] : kNotEligible;
    hist_add(hist, key >> 20, key != kNotEligible);
  }
  __syncthreads();
  const int n_elig = rank_bins(hist, 2048, s_budget, s_warp, &s_bin, &s_k);
  const int budget = min(s_budget, n_elig);
  uint32_t thr = 0x80000000u;  // above every eligible key: nothing selected
  int take_eq = 0;
  if (budget > 0) {
    uint32_t prefix = uint32_t(s_bin) << 20;
    for (int i = tid; i < 2048; i += kThreads) hist[i] = 0u;
    __syncthreads();
    for (int base = warp * 32; base < n; base += kThreads) {
      const int p = base + lane;
      const uint32_t key = p < n ? keys[p] : kNotEligible;
      hist_add(hist, (key >> 9) & 0x7ffu, (key >> 20) == (prefix >> 20));
    }
    __syncthreads();
    rank_bins(hist, 2048, s_k, s_warp, &s_bin, &s_k);
    prefix |= uint32_t(s_bin) << 9;
    for (int i = tid; i < 512; i += kThreads) hist[i] = 0u;
    __syncthreads();
    for (int base = warp * 32; base < n; base += kThreads) {
      const int p = base + lane;
      const uint32_t key = p < n ? keys[p] : kNotEligible;
      hist_add(hist, key & 0x1ffu, (key >> 9) == (prefix >> 9));
    }
    __syncthreads();
    rank_bins(hist, 512, s_k, s_warp, &s_bin, &s_k);
    thr = prefix | uint32_t(s_bin);
    take_eq = s_k;
  }

  // 5. mark: keys above thr, then the first take_eq equal to it by position; compact
  // (torch_engine.py:144-150).  Each thread owns one contiguous run of positions.
  const int seg = (n + kThreads - 1) / kThreads;
  const int p0 = min(n, tid * seg), p1 = min(n, p0 + seg);
  int c_eq = 0;
  if (take_eq > 0)
    for (int p = p0; p < p1; ++p) c_eq += keys[p] == thr ? 1 : 0;
  int4 tot;
  int r = block_scan4(make_int4(c_eq, 0, 0, 0), &tot, s_warp).x;
  int4 c = make_int4(0, 0, 0, 0);  // kept, exact, kept & cached, kept & exact
  for (int p = p0; p < p1; ++p) {
    const uint32_t key = keys[p];
    uint8_t f = fl[p];
    bool kept;
    if (key != kNotEligible) {
      kept = key > thr;
      if (key == thr) kept = r++ < take_eq;
    } else {
      kept = (f & kKeep) != 0;
    }
    if (kept) {
      f |= kKept;
      fl[p] = f;
      ++c.x;
      if (f & kCached) ++c.z;
      if (f & kExact) ++c.w;
    }
    if (f & kExact) ++c.y;
  }
  const int4 base = block_scan4(c, &tot, s_warp);
  int out = base.x, ex = base.y;
  for (int p = p0; p < p1; ++p) {
    const uint8_t f = fl[p];
    if (f & kKept) {
      a.keep_abs[out] = p;
      a.sel[out] = p - ex;
      ++out;
    }
    if (f & kExact) ++ex;
  }
  if (tid == 0) {
    const int n_sel = tot.x, sel_cached = tot.z, bad = tot.w;
    a.counts[0] = n_sel;
    a.counts[1] = sel_cached;
    a.counts[2] = budget;
    a.counts[3] = n_elig;
    a.counts[4] = int(s_escmask);
    a.counts[5] = bad ? int(CKV_DEV_ERR_SELECT_UNCOMPUTED) : 0;
    a.counts[6] = n_sel - sel_cached;
    a.counts[7] = 0;
    if (bad) atomicOr(&g_err_word, CKV_DEV_ERR_SELECT_UNCOMPUTED);
  }
}

// Phase 1 for one active row i (one warp): diff[p], norm[p] for p = active[i].
__device__ __forceinline__ void deviation_row(
    int64_t i, const uint16_t* __restrict__ k_fresh, const uint16_t* __restrict__ v_fresh,
    int64_t fstride, const uint16_t* __restrict__ k_base, const uint16_t* __restrict__ v_base,
    const int32_t* __restrict__ active, int H, int D, const uint8_t* __restrict__ pos_flags,
    int n_ctx, float* diff, float* norm) {
  const int lane = threadIdx.x & 31;
  const int p = active[i];
  if (p < 0 || p >= n_ctx) {
    if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
    return;
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
  if (lane == 0) {
    diff[p] = dk + dv;
    norm[p] = nk + nv;
  }
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
__device__ __forceinline__ void deviation_rows(const RowArgs& r) {
  const int warp = threadIdx.x >> 5;
  const int64_t r0 = int64_t(blockIdx.x) * r.n_act / gridDim.x;
  const int64_t r1 = int64_t(blockIdx.x + 1) * r.n_act / gridDim.x;
  for (int64_t i = r0 + warp; i < r1; i += kWarps)
    deviation_row(i, r.k_fresh, r.v_fresh, r.fstride, r.k_base, r.v_base, r.active, r.H, r.D,
                  r.pos_flags, r.n_ctx, r.diff, r.norm);
}

__global__ void __launch_bounds__(kThreads) deviation_scores_kernel(RowArgs r) {
  deviation_rows(r);
}

__global__ void __launch_bounds__(kThreads) deviation_select_kernel(RowArgs r, unsigned* counter,
                                                                     SelectArgs sa) {
  extern __shared__ __align__(16) unsigned char dyn_smem[];
  __shared__ int s_last;
  deviation_rows(r);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(counter, 1u);
    s_last = (prev == gridDim.x - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const bool in_smem = sa.n_ctx <= kSmemPositions;
  uint32_t* keys = in_smem ? reinterpret_cast<uint32_t*>(dyn_smem) : sa.keys_scratch;
  uint8_t* fl = in_smem ? dyn_smem + 4 * size_t(sa.n_ctx) : sa.flags_scratch;
  select_tail(sa, keys, fl);
  if (threadIdx.x == 0) *counter = 0u;  // ready for the next launch
}

__global__ void __launch_bounds__(kThreads) select_only_kernel(SelectArgs sa) {
  extern __shared__ __align__(16) unsigned char dyn_smem[];
  const bool in_smem = sa.n_ctx <= kSmemPositions;
  uint32_t* keys = in_smem ? reinterpret_cast<uint32_t*>(dyn_smem) : sa.keys_scratch;
  uint8_t* fl = in_smem ? dyn_smem + 4 * size_t(sa.n_ctx) : sa.flags_scratch;
  select_tail(sa, keys, fl);
}

int check_select(const uint8_t* pos_flags, int n_ctx, const int32_t* meta, int n_chunks,
                 float* rel, int32_t* keep_abs, int32_t* sel, int32_t* counts, uint8_t* scratch) {
  CKV_REQUIRE(pos_flags && rel && keep_abs && sel && counts && scratch,
              "selection: null pointer");
  CKV_REQUIRE(n_chunks == 0 || meta, "selection: null chunk table");
  CKV_REQUIRE(n_ctx > 0 && n_chunks >= 0, "selection: bad sizes");
  CKV_REQUIRE((reinterpret_cast<uintptr_t>(scratch) & 3u) == 0,
              "selection: scratch must be 4-byte aligned");
  return CKV_OK;
}

SelectArgs make_select_args(const float* diff, const float* norm, const uint8_t* pos_flags,
                            int n_ctx, const int32_t* meta, int n_chunks, int has_thr, double thr,
                            float* rel, int32_t* keep_abs, int32_t* sel, int32_t* counts,
                            uint8_t* scratch) {
  return SelectArgs{diff, norm, pos_flags, n_ctx, meta, n_chunks, has_thr, thr, rel, keep_abs,
                    sel, counts, reinterpret_cast<uint32_t*>(scratch), scratch + 4 * size_t(n_ctx)};
}

// Phase-1 grid: two 1024-thread CTAs per SM (every SM gets the same number of rows),
// at most one CTA per row.
int rows_grid(int n_act) { return std::max(1, std::min(n_act, 2 * num_sms())); }

int launch_fused(const RowArgs& r, unsigned* counter, const SelectArgs& sa, cudaStream_t st,
                 const char* name) {
  const int dyn = dyn_smem_bytes(sa.n_ctx);
  if (int rc = set_smem_limit(reinterpret_cast<const void*>(deviation_select_kernel),
                              dyn_smem_bytes(kSmemPositions)))
    return rc;
  deviation_select_kernel<<<rows_grid(r.n_act), kThreads, dyn, st>>>(r, counter, sa);
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
                         uint32_t* counter, ckv_stream_t stream) {
  if (int rc = check_select(pos_flags, n_ctx, sel_meta, n_chunks, rel, keep_abs, sel, counts,
                            scratch))
    return rc;
  CKV_REQUIRE(k_fresh && v_fresh && k_base && v_base && active && diff && norm && counter,
              "ckv_deviation_select: null pointer");
  CKV_REQUIRE(aligned16(k_fresh) && aligned16(v_fresh) && aligned16(k_base) && aligned16(v_base),
              "ckv_deviation_select: K/V must be 16-byte aligned");
  CKV_REQUIRE(head_dim % 8 == 0 && fresh_row_stride % 8 == 0 && n_kv_heads > 0,
              "ckv_deviation_select: head_dim and row stride must be multiples of 8");
  CKV_REQUIRE(n_act > 0 && n_act <= n_ctx, "ckv_deviation_select: n_act %d out of range", n_act);
  const RowArgs r{k_fresh, v_fresh, fresh_row_stride, k_base, v_base, active, n_act,
                  n_kv_heads, head_dim, pos_flags, n_ctx, diff, norm};
  const SelectArgs sa = make_select_args(diff, norm, pos_flags, n_ctx, sel_meta, n_chunks,
                                         has_threshold, escalate_threshold, rel, keep_abs, sel,
                                         counts, scratch);
  return launch_fused(r, counter, sa, as_stream(stream), "ckv_deviation_select");
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
                              dyn_smem_bytes(kSmemPositions)))
    return rc;
  select_only_kernel<<<1, kThreads, dyn_smem_bytes(n_ctx), as_stream(stream)>>>(sa);
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
// output buffers but no allocator to make the selection's two scratch buffers
// with.  For them the scratch lives here, in one file-scope device array that
// every GPU which loads the library keeps until the process exits:
//   bytes [0, 4)                                 the last-CTA ticket counter
//   bytes [256, 256 + 5 * CKV_NOALLOC_MAX_CTX)   the selection's per-position keys
//                                                and flags (phase 2 uses them only
//                                                when n_ctx exceeds what it keeps
//                                                in shared memory)
// Its device address is looked up once per device (cudaGetSymbolAddress, on the
// first call made while that device is current).  Every call shares the array:
// the counter is cleared with an async memset on the caller's stream before
// each launch and the keys and flags are rewritten in full, but two calls that
// overlap on the GPU (different streams, no ordering between them) race on it.
#include <atomic>

namespace ckv {
namespace {

constexpr int kNoAllocScratchOffset = 256;
static __device__ __align__(256) unsigned char
    g_noalloc_scratch[kNoAllocScratchOffset + 5 * CKV_NOALLOC_MAX_CTX];

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
  uint32_t* counter = reinterpret_cast<uint32_t*>(scratch);
  uint8_t* select_scratch = scratch + kNoAllocScratchOffset;
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
  // the ticket counter must start at zero; a memset is a copy, not an allocation
  cudaError_t e = cudaMemsetAsync(counter, 0, sizeof(uint32_t), as_stream(stream));
  if (e != cudaSuccess) {
    set_error("ckv_deviation_select_noalloc: clearing the counter failed: %s", cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  const RowArgs r{k_fresh, v_fresh, fresh_row_stride, k_base, v_base, active, n_act,
                  n_kv_heads, head_dim, pos_flags, n_ctx, diff, norm};
  const SelectArgs sa = make_select_args(diff, norm, pos_flags, n_ctx, sel_meta, n_chunks,
                                         has_threshold, escalate_threshold, rel, keep_abs, sel,
                                         counts, select_scratch);
  return launch_fused(r, counter, sa, as_stream(stream), "ckv_deviation_select_noalloc");
}
