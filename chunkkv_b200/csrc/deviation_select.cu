// Layer-1 K/V deviation + pooled top-k selection (torch_engine.py:117-153).
//
// One launch.  Phase 1 (every CTA): one warp per active token computes
//   diff = sum_{h,d} fp32(bf16(k - K))^2 + sum fp32(bf16(v - V))^2   (torch_engine.py:118-119)
//   norm = sum fp32(k)^2 + sum fp32(v)^2                             (torch_engine.py:120)
// Phase 2 (the last CTA to finish, found with an atomic ticket — no waiting):
//   per-chunk rel = sum diff / sum norm over the chunk span           (torch_engine.py:132)
//   keep = ~cached | sink | escalated spans; pool = pooled spans     (torch_engine.py:125-140)
//   budget = min(sum of per-chunk budgets, |pool & ~keep|)          (torch_engine.py:139,142)
//   top-`budget` eligible positions by diff (radix select on the fp32 bit
//   pattern, diff >= 0; equal scores: lower position first — the reference's
//   argsort leaves that order undefined, torch_engine.py:144)
//   keep_abs = ascending kept positions, sel = index in the active list (146-150).
#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(select)

namespace ckv {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

// pos_flags input bits
constexpr uint8_t kInCached = 1, kInSink = 2, kInExact = 4;
// working flag bits (scratch)
constexpr uint8_t kKeep = 1, kPool = 2, kExact = 4, kCached = 8;

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
  uint8_t* flags;
};

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

// Block-wide exclusive scan of two ints (all kThreads threads call it).
__device__ int2 block_exclusive_scan2(int a, int b, int2* total, int2* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ta = __shfl_up_sync(0xffffffffu, ia, o);
    const int tb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ta;
      ib += tb;
    }
  }
  if (lane == 31) s_warp[warp] = make_int2(ia, ib);
  __syncthreads();
  if (warp == 0) {
    int2 w = lane < kWarps ? s_warp[lane] : make_int2(0, 0);
    int wa = w.x, wb = w.y;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ta = __shfl_up_sync(0xffffffffu, wa, o);
      const int tb = __shfl_up_sync(0xffffffffu, wb, o);
      if (lane >= o) {
        wa += ta;
        wb += tb;
      }
    }
    if (lane < kWarps) s_warp[lane] = make_int2(wa - w.x, wb - w.y);  // exclusive
    if (lane == kWarps - 1) s_warp[kWarps] = make_int2(wa, wb);      // block total
  }
  __syncthreads();
  const int2 base = s_warp[warp];
  *total = s_warp[kWarps];
  __syncthreads();  // s_warp reusable after return
  return make_int2(base.x + ia - a, base.y + ib - b);
}

__device__ int block_sum(int v, int* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_i(v);
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kWarps ? s_red[lane] : 0;
    w = warp_sum_i(w);
    if (lane == 0) s_red[kWarps] = w;
  }
  __syncthreads();
  const int t = s_red[kWarps];
  __syncthreads();
  return t;
}

__device__ __forceinline__ bool eligible(uint8_t f) { return (f & kPool) && !(f & kKeep); }

// Phase 2: the selection, run by one CTA of kThreads threads.
__device__ void select_phase(const SelectArgs& a) {
  __shared__ unsigned hist[256];
  __shared__ int2 s_scan[kWarps + 1];
  __shared__ int s_red[kWarps + 1];
  __shared__ int s_budget;
  __shared__ int s_digit, s_k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = a.n_ctx;

  // 1. initial flags: keep = ~cached | sink (torch_engine.py:125)
  for (int p = tid; p < n; p += kThreads) {
    const uint8_t f = a.pos_flags[p];
    uint8_t w = 0;
    if (!(f & kInCached) || (f & kInSink)) w |= kKeep;
    if (f & kInExact) w |= kExact;
    if (f & kInCached) w |= kCached;
    a.flags[p] = w;
  }
  if (tid == 0) s_budget = 0;
  __syncthreads();

  // 2. per-chunk rel, escalation, pool, budget (torch_engine.py:128-140)
  for (int c = warp; c < a.n_chunks; c += kWarps) {
    const int32_t* m = a.meta + c * CKV_SEL_META_STRIDE;
    const int start = m[0], len = m[1], budget_c = m[2], exact = m[3];
    if (exact) continue;
    float sd = 0.f, sn = 0.f;
    for (int p = start + lane; p < start + len; p += 32) {
      if (p >= 0 && p < n) {
        sd += __ldcg(a.diff + p);
        sn += __ldcg(a.norm + p);
      }
    }
    sd = warp_sum(sd);
    sn = warp_sum(sn);
    const float rel = __fdiv_rn(sd, sn);
    const bool esc = a.has_thr && (double(rel) > a.thr);
    if (lane == 0) a.rel[c] = rel;
    if (esc || budget_c >= 0) {
      const unsigned bit = esc ? kKeep : kPool;
      for (int p = start + lane; p < start + len; p += 32) {
        if (p < 0 || p >= n) continue;
        unsigned* word = reinterpret_cast<unsigned*>(a.flags + (p & ~3));
        atomicOr(word, bit << (8 * (p & 3)));
      }
      if (!esc && lane == 0) atomicAdd(&s_budget, budget_c);
    }
  }
  __syncthreads();

  // 3. eligible count and budget cap (torch_engine.py:142)
  int local = 0;
  for (int p = tid; p < n; p += kThreads) local += eligible(a.flags[p]) ? 1 : 0;
  const int n_elig = block_sum(local, s_red);
  const int budget = min(s_budget, n_elig);

  // 4. radix select of the budget-th largest diff among eligible positions
  unsigned prefix = 0, mask = 0;
  int k = budget;
  if (budget > 0) {
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
      __syncthreads();
      for (int p = tid; p < n; p += kThreads) {
        if (!eligible(a.flags[p])) continue;
        const unsigned key = __float_as_uint(__ldcg(a.diff + p));
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (warp == 0) {
        // lane owns digits 255-8*lane .. 248-8*lane (descending)
        int cnt[8], sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          cnt[i] = hist[255 - (lane * 8 + i)];
          sum += cnt[i];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        const int excl = incl - sum;
        const unsigned hit = __ballot_sync(0xffffffffu, incl >= k);
        const int first = __ffs(hit) - 1;  // lane whose range crosses k
        if (lane == first) {
          int cum = excl;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (cum + cnt[i] >= k) {
              s_digit = 255 - (lane * 8 + i);
              s_k = k - cum;
              break;
            }
            cum += cnt[i];
          }
        }
      }
      __syncthreads();
      prefix |= unsigned(s_digit) << shift;
      mask |= 255u << shift;
      k = s_k;
      __syncthreads();
    }
  }
  const unsigned thr_key = prefix;  // value of the budget-th largest
  const int take_eq = budget > 0 ? k : 0;

  // 5. mark selected: key > thr_key, plus the first take_eq (by position) equal to it
  const int seg = (n + kThreads - 1) / kThreads;
  const int p0 = min(n, tid * seg), p1 = min(n, p0 + seg);
  int c_eq = 0;
  if (budget > 0)
    for (int p = p0; p < p1; ++p)
      if (eligible(a.flags[p]) && __float_as_uint(__ldcg(a.diff + p)) == thr_key) ++c_eq;
  int2 tot;
  const int2 base_eq = block_exclusive_scan2(c_eq, 0, &tot, s_scan);
  if (budget > 0) {
    int r = base_eq.x;
    for (int p = p0; p < p1; ++p) {
      const uint8_t f = a.flags[p];
      if (!eligible(f)) continue;
      const unsigned key = __float_as_uint(__ldcg(a.diff + p));
      bool take = key > thr_key;
      if (key == thr_key) {
        take = r < take_eq;
        ++r;
      }
      if (take) a.flags[p] = f | kKeep;
    }
  }

  // 6. compaction (torch_engine.py:146-150) and counts
  int c_keep = 0, c_exact = 0, c_cached = 0, c_bad = 0;
  for (int p = p0; p < p1; ++p) {
    const uint8_t f = a.flags[p];
    if (f & kKeep) {
      ++c_keep;
      if (f & kCached) ++c_cached;
      if (f & kExact) ++c_bad;
    }
    if (f & kExact) ++c_exact;
  }
  const int2 base = block_exclusive_scan2(c_keep, c_exact, &tot, s_scan);
  const int n_sel = tot.x;
  int out = base.x, ex = base.y;
  for (int p = p0; p < p1; ++p) {
    const uint8_t f = a.flags[p];
    if (f & kKeep) {
      a.keep_abs[out] = p;
      a.sel[out] = p - ex;
      ++out;
    }
    if (f & kExact) ++ex;
  }
  const int sel_cached = block_sum(c_cached, s_red);
  const int bad = block_sum(c_bad, s_red);
  if (tid == 0) {
    a.counts[0] = n_sel;
    a.counts[1] = sel_cached;
    a.counts[2] = budget;
    a.counts[3] = n_elig;
    a.counts[4] = 0;
    a.counts[5] = bad ? int(CKV_DEV_ERR_SELECT_UNCOMPUTED) : 0;
    a.counts[6] = n_sel - sel_cached;
    a.counts[7] = 0;
    if (bad) atomicOr(&g_err_word, CKV_DEV_ERR_SELECT_UNCOMPUTED);
  }
}

// Phase 1: one warp per active token; writes diff[p], norm[p] for p = active[i].
__device__ __forceinline__ void deviation_rows(
    const uint16_t* __restrict__ k_fresh, const uint16_t* __restrict__ v_fresh, int64_t fstride,
    const uint16_t* __restrict__ k_base, const uint16_t* __restrict__ v_base,
    const int32_t* __restrict__ active, int n_act, int H, int D, const uint8_t* __restrict__ pos_flags,
    int n_ctx, float* diff, float* norm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int vecs = (H * D) / 8;
  for (int i = blockIdx.x * kWarps + warp; i < n_act; i += gridDim.x * kWarps) {
    const int p = active[i];
    if (p < 0 || p >= n_ctx) {
      if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
      continue;
    }
    // the reference compares against a zero-initialised cache (torch_engine.py:97) that
    // only moved chunks fill, so a position no chunk covers compares against zeros
    const bool cached = (pos_flags[p] & kInCached) != 0;
    float dk = 0.f, dv = 0.f, nk = 0.f, nv = 0.f;
    for (int v = lane; v < vecs; v += 32) {
      const int e0 = v * 8, h = e0 / D, d = e0 - h * D;
      const int64_t boff = (int64_t(h) * n_ctx + p) * D + d;
      const uint4 kf = *reinterpret_cast<const uint4*>(k_fresh + i * fstride + e0);
      const uint4 vf = *reinterpret_cast<const uint4*>(v_fresh + i * fstride + e0);
      const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
      const uint4 kb = cached ? *reinterpret_cast<const uint4*>(k_base + boff) : zero;
      const uint4 vb = cached ? *reinterpret_cast<const uint4*>(v_base + boff) : zero;
      const uint32_t* pkf = reinterpret_cast<const uint32_t*>(&kf);
      const uint32_t* pvf = reinterpret_cast<const uint32_t*>(&vf);
      const uint32_t* pkb = reinterpret_cast<const uint32_t*>(&kb);
      const uint32_t* pvb = reinterpret_cast<const uint32_t*>(&vb);
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
    dk = warp_sum(dk);
    dv = warp_sum(dv);
    nk = warp_sum(nk);
    nv = warp_sum(nv);
    if (lane == 0) {
      diff[p] = dk + dv;
      norm[p] = nk + nv;
    }
  }
}

__global__ void __launch_bounds__(kThreads) deviation_scores_kernel(
    const uint16_t* __restrict__ k_fresh, const uint16_t* __restrict__ v_fresh, int64_t fstride,
    const uint16_t* __restrict__ k_base, const uint16_t* __restrict__ v_base,
    const int32_t* __restrict__ active, int n_act, int H, int D, const uint8_t* __restrict__ pos_flags,
    int n_ctx, float* diff, float* norm) {
  deviation_rows(k_fresh, v_fresh, fstride, k_base, v_base, active, n_act, H, D, pos_flags, n_ctx,
                 diff, norm);
}

__global__ void __launch_bounds__(kThreads) deviation_select_kernel(
    const uint16_t* __restrict__ k_fresh, const uint16_t* __restrict__ v_fresh, int64_t fstride,
    const uint16_t* __restrict__ k_base, const uint16_t* __restrict__ v_base,
    const int32_t* __restrict__ active, int n_act, int H, int D, float* diff, float* norm,
    unsigned* counter, SelectArgs sa) {
  __shared__ int s_last;
  deviation_rows(k_fresh, v_fresh, fstride, k_base, v_base, active, n_act, H, D, sa.pos_flags,
                 sa.n_ctx, diff, norm);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(counter, 1u);
    s_last = (prev == gridDim.x - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  select_phase(sa);
  if (threadIdx.x == 0) *counter = 0u;  // ready for the next launch
}

__global__ void __launch_bounds__(kThreads) select_only_kernel(SelectArgs sa) { select_phase(sa); }

int check_select(const uint8_t* pos_flags, int n_ctx, const int32_t* meta, int n_chunks,
                 float* rel, int32_t* keep_abs, int32_t* sel, int32_t* counts, uint8_t* flags) {
  CKV_REQUIRE(pos_flags && rel && keep_abs && sel && counts && flags,
              "selection: null pointer");
  CKV_REQUIRE(n_chunks == 0 || meta, "selection: null chunk table");
  CKV_REQUIRE(n_ctx > 0 && n_chunks >= 0, "selection: bad sizes");
  CKV_REQUIRE((reinterpret_cast<uintptr_t>(flags) & 3u) == 0,
              "selection: flags scratch must be 4-byte aligned");
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
                         int32_t* keep_abs, int32_t* sel, int32_t* counts, uint8_t* flags,
                         uint32_t* counter, ckv_stream_t stream) {
  if (int rc = check_select(pos_flags, n_ctx, sel_meta, n_chunks, rel, keep_abs, sel, counts, flags))
    return rc;
  CKV_REQUIRE(k_fresh && v_fresh && k_base && v_base && active && diff && norm && counter,
              "ckv_deviation_select: null pointer");
  CKV_REQUIRE(aligned16(k_fresh) && aligned16(v_fresh) && aligned16(k_base) && aligned16(v_base),
              "ckv_deviation_select: K/V must be 16-byte aligned");
  CKV_REQUIRE(head_dim % 8 == 0 && fresh_row_stride % 8 == 0 && n_kv_heads > 0,
              "ckv_deviation_select: head_dim and row stride must be multiples of 8");
  CKV_REQUIRE(n_act > 0 && n_act <= n_ctx, "ckv_deviation_select: n_act %d out of range", n_act);
  SelectArgs sa{diff, norm, pos_flags, n_ctx, sel_meta, n_chunks, has_threshold,
                escalate_threshold, rel, keep_abs, sel, counts, flags};
  const int grid = std::min(ceil_div(n_act, kWarps), 2 * num_sms());
  deviation_select_kernel<<<grid, kThreads, 0, as_stream(stream)>>>(
      k_fresh, v_fresh, fresh_row_stride, k_base, v_base, active, n_act, n_kv_heads, head_dim,
      diff, norm, counter, sa);
  CKV_LAUNCH_CHECK("ckv_deviation_select");
  return CKV_OK;
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
  const int grid = std::min(ceil_div(n_act, kWarps), 2 * num_sms());
  deviation_scores_kernel<<<grid, kThreads, 0, as_stream(stream)>>>(
      k_fresh, v_fresh, fresh_row_stride, k_base, v_base, active, n_act, n_kv_heads, head_dim,
      pos_flags, n_ctx, diff, norm);
  CKV_LAUNCH_CHECK("ckv_deviation_scores");
  return CKV_OK;
}

int ckv_select_from_scores(const float* diff, const float* norm, const uint8_t* pos_flags,
                           int n_ctx, const int32_t* sel_meta, int n_chunks, int has_threshold,
                           double escalate_threshold, float* rel, int32_t* keep_abs,
                           int32_t* sel, int32_t* counts, uint8_t* flags, ckv_stream_t stream) {
  if (int rc = check_select(pos_flags, n_ctx, sel_meta, n_chunks, rel, keep_abs, sel, counts, flags))
    return rc;
  CKV_REQUIRE(diff && norm, "ckv_select_from_scores: null scores");
  SelectArgs sa{diff, norm, pos_flags, n_ctx, sel_meta, n_chunks, has_threshold,
                escalate_threshold, rel, keep_abs, sel, counts, flags};
  select_only_kernel<<<1, kThreads, 0, as_stream(stream)>>>(sa);
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
//   bytes [0, 4)                      the last-CTA ticket counter
//   bytes [256, 256 + CKV_NOALLOC_MAX_CTX)  one flag byte per position
// Its device address is looked up once per device (cudaGetSymbolAddress, on the
// first call made while that device is current).  Every call shares the array:
// the counter is cleared with an async memset on the caller's stream before
// each launch and the flags are rewritten in full, but two calls that overlap
// on the GPU (different streams, no ordering between them) race on it.
namespace ckv {
namespace {

constexpr int kNoAllocFlagsOffset = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocFlagsOffset + CKV_NOALLOC_MAX_CTX];

constexpr int kNoAllocMaxDevices = 64;

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int noalloc_scratch(unsigned char** out) {
  static unsigned char* addr[kNoAllocMaxDevices] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    set_error("ckv_deviation_select_noalloc: no usable current device (%s)", cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("ckv_deviation_select_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return CKV_ERR_CUDA;
    }
    addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = addr[dev];
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
  uint8_t* flags = scratch + kNoAllocFlagsOffset;
  if (int rc = check_select(pos_flags, n_ctx, sel_meta, n_chunks, rel, keep_abs, sel, counts, flags))
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
  SelectArgs sa{diff, norm, pos_flags, n_ctx, sel_meta, n_chunks, has_threshold,
                escalate_threshold, rel, keep_abs, sel, counts, flags};
  const int grid = std::min(ceil_div(n_act, kWarps), 2 * num_sms());
  deviation_select_kernel<<<grid, kThreads, 0, as_stream(stream)>>>(
      k_fresh, v_fresh, fresh_row_stride, k_base, v_base, active, n_act, n_kv_heads, head_dim,
      diff, norm, counter, sa);
  CKV_LAUNCH_CHECK("ckv_deviation_select_noalloc");
  return CKV_OK;
}
