// Bandwidth-bound pieces of the recompute: embedding rows, RMSNorm, the
// shrink-to-selection copy/scatter, the small-m lm_head projection and the
// final log-softmax (one 8-CTA cluster per row).  Row copies are 16-byte vectorised, one warp or CTA per row.
#include <cooperative_groups.h>

#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(elementwise)

namespace ckv {
namespace {

namespace cg = cooperative_groups;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// out[i] = table[tokens[rows[i]]]   (torch_engine.py:105-107)
__global__ void embed_kernel(const uint16_t* __restrict__ table, int vocab, int hidden,
                             const int32_t* __restrict__ tokens, const int32_t* __restrict__ rows,
                             int n_rows, uint16_t* __restrict__ out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int vecs = hidden / 8;
  for (int i = warp; i < n_rows; i += nw) {
    const int tok = tokens[rows ? rows[i] : i];
    if (tok < 0 || tok >= vocab) {
      if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(table + int64_t(tok) * hidden);
    uint4* dst = reinterpret_cast<uint4*>(out + int64_t(i) * hidden);
    for (int v = lane; v < vecs; v += 32) dst[v] = src[v];
  }
}

// Qwen2RMSNorm: y = w * bf16(x * rsqrt(mean(x^2) + eps)), fp32 inside.
// One 128-thread CTA per row; each thread keeps its (at most kRmsVec) 16-byte vectors
// of the row in registers between the reduction and the write, so x is read once.
// kAdd: first h = bf16(h + delta) (the residual add of a row-parallel projection whose
// partial sums were all-reduced), written back to h, then y = RMSNorm(h).
constexpr int kRmsThreads = 128;
constexpr int kRmsVec = 5;  // hidden <= 128 * 8 * 5 = 5120
template <bool kAdd>
__global__ void __launch_bounds__(kRmsThreads) rmsnorm_kernel(uint16_t* __restrict__ x,
                                                              const uint16_t* __restrict__ delta,
                                                              const uint16_t* __restrict__ w,
                                                              uint16_t* __restrict__ y, int hidden,
                                                              float eps) {
  __shared__ float s_red[kRmsThreads / 32];
  pdl_wait();  // h comes from the kernel before (dependent launch)
  pdl_launch_next();
  const int row = blockIdx.x;
  uint4* xr = reinterpret_cast<uint4*>(x + int64_t(row) * hidden);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + int64_t(row) * hidden);
  const int vecs = hidden / 8;
  // the row and the weight are requested together: one memory latency, not two
  uint4 v[kRmsVec], wv[kRmsVec];
#pragma unroll
  for (int i = 0; i < kRmsVec; ++i) {
    const int c = threadIdx.x + kRmsThreads * i;
    v[i] = c < vecs ? __ldcs(xr + c) : make_uint4(0u, 0u, 0u, 0u);
    wv[i] = c < vecs ? __ldg(wr + c) : make_uint4(0u, 0u, 0u, 0u);
  }
  if constexpr (kAdd) {
    const uint4* dr = reinterpret_cast<const uint4*>(delta + int64_t(row) * hidden);
#pragma unroll
    for (int i = 0; i < kRmsVec; ++i) {
      const int c = threadIdx.x + kRmsThreads * i;
      if (c < vecs) {
        const uint4 dv = __ldcs(dr + c);
        uint32_t* p = reinterpret_cast<uint32_t*>(&v[i]);
        const uint32_t* q = reinterpret_cast<const uint32_t*>(&dv);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          p[e] = pack_bf2(__fadd_rn(lo_bf(p[e]), lo_bf(q[e])), __fadd_rn(hi_bf(p[e]), hi_bf(q[e])));
        xr[c] = v[i];
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kRmsVec; ++i) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(&v[i]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float f0 = lo_bf(p[e]), f1 = hi_bf(p[e]);
      ss = __fadd_rn(ss, __fmul_rn(f0, f0));
      ss = __fadd_rn(ss, __fmul_rn(f1, f1));
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float tot = (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]);
  const float r = rsqrtf(__fadd_rn(__fmul_rn(tot, 1.0f / float(hidden)), eps));
#pragma unroll
  for (int i = 0; i < kRmsVec; ++i) {
    const int c = threadIdx.x + kRmsThreads * i;
    if (c < vecs) {
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&v[i]);
      const uint32_t* q = reinterpret_cast<const uint32_t*>(&wv[i]);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float n0 = bf16_round(__fmul_rn(lo_bf(p[e]), r));
        const float n1 = bf16_round(__fmul_rn(hi_bf(p[e]), r));
        po[e] = pack_bf2(__fmul_rn(lo_bf(q[e]), n0), __fmul_rn(hi_bf(q[e]), n1));
      }
      yr[c] = o;
    }
  }
}

// Shrink h/x to the selected rows and write their fresh k/v into the cache.
__global__ void apply_selection_kernel(const int32_t* __restrict__ sel,
                                       const int32_t* __restrict__ keep_abs,
                                       const int32_t* __restrict__ counts, int max_rows,
                                       const uint16_t* __restrict__ h_in, uint16_t* __restrict__ h_out,
                                       const uint16_t* __restrict__ x_in, uint16_t* __restrict__ x_out,
                                       int hidden, const uint16_t* __restrict__ k_fresh,
                                       const uint16_t* __restrict__ v_fresh, int64_t fstride,
                                       uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache,
                                       int H, int D, int n_ctx) {
  const int n_sel = min(counts[0], max_rows);
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int hv = hidden / 8, kvv = (H * D) / 8;
  for (int i = warp; i < n_sel; i += nw) {
    const int src = sel[i];
    const int pos = keep_abs[i];
    if (pos < 0 || pos >= n_ctx || src < 0 || src >= max_rows) {
      if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
      continue;
    }
    const uint4* hs = reinterpret_cast<const uint4*>(h_in + int64_t(src) * hidden);
    const uint4* xs = reinterpret_cast<const uint4*>(x_in + int64_t(src) * hidden);
    uint4* hd = reinterpret_cast<uint4*>(h_out + int64_t(i) * hidden);
    uint4* xd = reinterpret_cast<uint4*>(x_out + int64_t(i) * hidden);
    for (int v = lane; v < hv; v += 32) {
      hd[v] = hs[v];
      xd[v] = xs[v];
    }
    for (int v = lane; v < kvv; v += 32) {
      const int e0 = v * 8, h = e0 / D, d = e0 - h * D;
      const int64_t coff = (int64_t(h) * n_ctx + pos) * D + d;
      *reinterpret_cast<uint4*>(k_cache + coff) =
          *reinterpret_cast<const uint4*>(k_fresh + src * fstride + e0);
      *reinterpret_cast<uint4*>(v_cache + coff) =
          *reinterpret_cast<const uint4*>(v_fresh + src * fstride + e0);
    }
  }
}

// out[m][n] = bf16(sum_k x[m][k] * w[n][k]) for m <= 8; one warp per weight row.
template <int MM>
__global__ void __launch_bounds__(256) gemv_kernel(const uint16_t* __restrict__ x,
                                                   const uint16_t* __restrict__ w,
                                                   uint16_t* __restrict__ out, int n, int k) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= n) return;
  const uint4* wr = reinterpret_cast<const uint4*>(w + int64_t(warp) * k);
  const int vecs = k / 8;
  float acc[MM];
#pragma unroll
  for (int m = 0; m < MM; ++m) acc[m] = 0.f;
  for (int v = lane; v < vecs; v += 32) {
    const uint4 a = __ldcs(wr + v);  // streamed once
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
    for (int m = 0; m < MM; ++m) {
      const uint4 b = reinterpret_cast<const uint4*>(x + int64_t(m) * k)[v];
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[m] = fmaf(lo_bf(pa[e]), lo_bf(pb[e]), acc[m]);
        acc[m] = fmaf(hi_bf(pa[e]), hi_bf(pb[e]), acc[m]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MM; ++m) {
    const float s = warp_sum(acc[m]);
    if (lane == 0) out[int64_t(m) * n + warp] = f2bf(s);
  }
}

// log_softmax of one row (float math, bf16 input) on one cluster of kLsmCtas CTAs.
// CTA r owns the contiguous slice [r * per, (r + 1) * per) of the row.  Each CTA
// publishes its slice's max, then its slice's sum of exp(x - max), in its own shared
// memory; every CTA reads the kLsmCtas partials through distributed shared memory and
// combines them in rank order, so all CTAs hold the same max and log-sum-exp and the
// result does not depend on timing.  The third pass writes (x - max) - lse.
constexpr int kLsmCtas = 8;
constexpr int kLsmThreads = 1024;
__device__ __forceinline__ float lsm_block_reduce(float v, bool is_max, float* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = is_max ? warp_max(v) : warp_sum(v);
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = s_red[lane];  // kLsmThreads / 32 == 32 partials
    t = is_max ? warp_max(t) : warp_sum(t);
    if (lane == 0) s_red[32] = t;
  }
  __syncthreads();
  const float r = s_red[32];
  __syncthreads();  // s_red is reused by the next reduction
  return r;
}
__global__ void __cluster_dims__(kLsmCtas, 1, 1) __launch_bounds__(kLsmThreads)
    log_softmax_kernel(const uint16_t* __restrict__ x, int n, float* __restrict__ out) {
  static_assert(kLsmThreads == 1024, "lsm_block_reduce assumes 32 warps");
  __shared__ float s_red[33];
  __shared__ float s_part[2];  // this CTA's slice max, then its slice sum
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = int(cluster.block_rank());
  const int per = (n + kLsmCtas - 1) / kLsmCtas;
  const int lo = min(n, rank * per), hi = min(n, lo + per);
  float mx = -INFINITY;
  for (int i = lo + int(threadIdx.x); i < hi; i += kLsmThreads) mx = fmaxf(mx, bf2f(x[i]));
  mx = lsm_block_reduce(mx, true, s_red);
  if (threadIdx.x == 0) s_part[0] = mx;
  cluster.sync();
  float gmax = -INFINITY;
#pragma unroll
  for (int q = 0; q < kLsmCtas; ++q) gmax = fmaxf(gmax, cluster.map_shared_rank(s_part, q)[0]);
  float sum = 0.f;
  for (int i = lo + int(threadIdx.x); i < hi; i += kLsmThreads) sum += expf(bf2f(x[i]) - gmax);
  sum = lsm_block_reduce(sum, false, s_red);
  if (threadIdx.x == 0) s_part[1] = sum;
  cluster.sync();
  float total = 0.f;
#pragma unroll
  for (int q = 0; q < kLsmCtas; ++q) total += cluster.map_shared_rank(s_part, q)[1];
  const float lse = logf(total);
  // No CTA may leave while another still reads its s_part: arrive now, wait at the end.
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  for (int i = lo + int(threadIdx.x); i < hi; i += kLsmThreads) out[i] = (bf2f(x[i]) - gmax) - lse;
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Greedy next token of the decode loop (logits[-1].argmax() and pos += 1,
// torch_engine.py:185,196-197): the argmax of one bf16 logits row on one cluster of
// kLsmCtas CTAs, each reducing one contiguous slice.  Order: NaN above every number
// (torch.argmax propagates NaN), then the larger value, and on equal values the lower
// index, so the result is torch.argmax's.  Rank 0 merges the slices' winners in rank
// order, writes the token id and, when `pos` is given, advances the decode position by
// one, so a replayed decode step needs no further kernel for either.
__device__ __forceinline__ bool argmax_better(float av, int ai, float bv, int bi) {
  const bool an = av != av, bn = bv != bv;
  if (an != bn) return an;
  if (!an && av != bv) return av > bv;
  return ai < bi;
}
__global__ void __cluster_dims__(kLsmCtas, 1, 1) __launch_bounds__(kLsmThreads)
    greedy_next_kernel(const uint16_t* __restrict__ x, int n, int32_t* __restrict__ tok,
                       int32_t* __restrict__ pos) {
  __shared__ float s_v[32];
  __shared__ int s_i[32];
  __shared__ float s_pv;  // this CTA's winner
  __shared__ int s_pi;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = int(cluster.block_rank());
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per = (n + kLsmCtas - 1) / kLsmCtas;
  const int lo = min(n, rank * per), hi = min(n, lo + per);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = lo + int(threadIdx.x); i < hi; i += kLsmThreads) {
    const float v = bf2f(x[i]);
    if (argmax_better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    s_v[warp] = bv;
    s_i[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    bv = s_v[lane];  // kLsmThreads / 32 == 32 warps
    bi = s_i[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (argmax_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      s_pv = bv;
      s_pi = bi;
    }
  }
  cluster.sync();
  if (rank == 0 && threadIdx.x == 0) {
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int q = 0; q < kLsmCtas; ++q) {
      const float qv = *cluster.map_shared_rank(&s_pv, q);
      const int qi = *cluster.map_shared_rank(&s_pi, q);
      if (argmax_better(qv, qi, v, idx)) {
        v = qv;
        idx = qi;
      }
    }
    tok[0] = idx;
    if (pos) pos[0] += 1;
  }
  cluster.sync();  // no CTA leaves while rank 0 still reads its winner
}

}  // namespace
}  // namespace ckv

using namespace ckv;

extern "C" {

int ckv_embed(const uint16_t* table, int vocab, int hidden, const int32_t* tokens,
              const int32_t* rows, int n_rows, uint16_t* out, ckv_stream_t stream) {
  CKV_REQUIRE(table && tokens && out, "ckv_embed: null pointer");
  CKV_REQUIRE(hidden > 0 && hidden % 8 == 0 && aligned16(table) && aligned16(out),
              "ckv_embed: hidden must be a multiple of 8 and rows 16-byte aligned");
  if (n_rows <= 0) return CKV_OK;
  const int grid = std::min(ceil_div(n_rows, 8), 8 * num_sms());
  embed_kernel<<<grid, 256, 0, as_stream(stream)>>>(table, vocab, hidden, tokens, rows, n_rows, out);
  CKV_LAUNCH_CHECK("ckv_embed");
  return CKV_OK;
}

int ckv_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows, int hidden, float eps,
                ckv_stream_t stream) {
  CKV_REQUIRE(x && w && y, "ckv_rmsnorm: null pointer");
  CKV_REQUIRE(hidden > 0 && hidden % 8 == 0 && aligned16(x) && aligned16(w) && aligned16(y),
              "ckv_rmsnorm: hidden must be a multiple of 8 and rows 16-byte aligned");
  CKV_REQUIRE(hidden <= kRmsThreads * 8 * kRmsVec, "ckv_rmsnorm: hidden %d above %d", hidden,
              kRmsThreads * 8 * kRmsVec);
  if (rows <= 0) return CKV_OK;
  launch_pdl(rmsnorm_kernel<false>, dim3(rows), dim3(kRmsThreads), 0, as_stream(stream),
             const_cast<uint16_t*>(x), static_cast<const uint16_t*>(nullptr), w, y, hidden, eps);
  CKV_LAUNCH_CHECK("ckv_rmsnorm");
  return CKV_OK;
}

int ckv_add_rmsnorm(uint16_t* h, const uint16_t* delta, const uint16_t* w, uint16_t* y, int rows,
                    int hidden, float eps, ckv_stream_t stream) {
  CKV_REQUIRE(h && delta && w && y, "ckv_add_rmsnorm: null pointer");
  CKV_REQUIRE(hidden > 0 && hidden % 8 == 0 && aligned16(h) && aligned16(delta) && aligned16(w) &&
                  aligned16(y),
              "ckv_add_rmsnorm: hidden must be a multiple of 8 and rows 16-byte aligned");
  CKV_REQUIRE(hidden <= kRmsThreads * 8 * kRmsVec, "ckv_add_rmsnorm: hidden %d above %d", hidden,
              kRmsThreads * 8 * kRmsVec);
  CKV_REQUIRE(y != h && y != delta, "ckv_add_rmsnorm: y must not alias h or delta");
  if (rows <= 0) return CKV_OK;
  launch_pdl(rmsnorm_kernel<true>, dim3(rows), dim3(kRmsThreads), 0, as_stream(stream), h, delta, w, y,
             hidden, eps);
  CKV_LAUNCH_CHECK("ckv_add_rmsnorm");
  return CKV_OK;
}

int ckv_apply_selection(const int32_t* sel, const int32_t* keep_abs, const int32_t* counts,
                        int max_rows, const uint16_t* h_in, uint16_t* h_out,
                        const uint16_t* x_in, uint16_t* x_out, int hidden,
                        const uint16_t* k_fresh, const uint16_t* v_fresh,
                        int64_t fresh_row_stride, uint16_t* k_cache, uint16_t* v_cache,
                        int n_kv_heads, int head_dim, int n_ctx, ckv_stream_t stream) {
  CKV_REQUIRE(sel && keep_abs && counts && h_in && h_out && x_in && x_out && k_fresh && v_fresh &&
                  k_cache && v_cache,
              "ckv_apply_selection: null pointer");
  CKV_REQUIRE(h_in != h_out && x_in != x_out, "ckv_apply_selection: in-place shrink not allowed");
  CKV_REQUIRE(hidden % 8 == 0 && head_dim % 8 == 0 && fresh_row_stride % 8 == 0,
              "ckv_apply_selection: sizes must be multiples of 8");
  CKV_REQUIRE(aligned16(h_in) && aligned16(h_out) && aligned16(x_in) && aligned16(x_out) &&
                  aligned16(k_fresh) && aligned16(v_fresh) && aligned16(k_cache) &&
                  aligned16(v_cache),
              "ckv_apply_selection: tensors must be 16-byte aligned");
  if (max_rows <= 0) return CKV_OK;
  const int grid = std::min(ceil_div(max_rows, 8), 8 * num_sms());
  apply_selection_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      sel, keep_abs, counts, max_rows, h_in, h_out, x_in, x_out, hidden, k_fresh, v_fresh,
      fresh_row_stride, k_cache, v_cache, n_kv_heads, head_dim, n_ctx);
  CKV_LAUNCH_CHECK("ckv_apply_selection");
  return CKV_OK;
}

int ckv_gemv(const uint16_t* x, const uint16_t* w, uint16_t* out, int m, int n, int k,
             ckv_stream_t stream) {
  CKV_REQUIRE(x && w && out, "ckv_gemv: null pointer");
  CKV_REQUIRE(m >= 1 && m <= 8, "ckv_gemv: m=%d outside 1..8", m);
  CKV_REQUIRE(k % 8 == 0 && aligned16(x) && aligned16(w), "ckv_gemv: k %% 8 and alignment");
  if (n <= 0) return CKV_OK;
  const int grid = ceil_div(n, 8);
  cudaStream_t s = as_stream(stream);
  switch (m) {
#define CKV_GEMV_CASE(MM) \
  case MM: gemv_kernel<MM><<<grid, 256, 0, s>>>(x, w, out, n, k); break;
    CKV_GEMV_CASE(1) CKV_GEMV_CASE(2) CKV_GEMV_CASE(3) CKV_GEMV_CASE(4)
    CKV_GEMV_CASE(5) CKV_GEMV_CASE(6) CKV_GEMV_CASE(7) CKV_GEMV_CASE(8)
#undef CKV_GEMV_CASE
  }
  CKV_LAUNCH_CHECK("ckv_gemv");
  return CKV_OK;
}

int ckv_greedy_next(const uint16_t* logits, int n, int32_t* token, int32_t* position, ckv_stream_t stream) {
  CKV_REQUIRE(logits && token && n > 0, "ckv_greedy_next: bad arguments");
  greedy_next_kernel<<<kLsmCtas, kLsmThreads, 0, as_stream(stream)>>>(logits, n, token, position);
  CKV_LAUNCH_CHECK("ckv_greedy_next");
  return CKV_OK;
}

int ckv_log_softmax(const uint16_t* logits, int n, float* out, ckv_stream_t stream) {
  CKV_REQUIRE(logits && out && n > 0, "ckv_log_softmax: bad arguments");
  log_softmax_kernel<<<kLsmCtas, kLsmThreads, 0, as_stream(stream)>>>(logits, n, out);
  CKV_LAUNCH_CHECK("ckv_log_softmax");
  return CKV_OK;
}

}  // extern "C"
