// Decode-time projections (m <= 8 rows): one warp per weight row (or row pair), the
// weight streamed from HBM once, with the same epilogues and rounding points as the
// tcgen05 GEMM's (gemm_tcgen05.cu): residual add, SwiGLU, and bias + RoPE + K/V cache
// scatter (torch_engine.py:61-76, 180-198 greedy decode).  At m <= 8 the GEMM's
// 128-row tiles would leave all but a handful of SMs idle on the 3584-column
// projections; here every SM streams weight rows.
#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(gemv_fused)

namespace ckv {
namespace {

constexpr int kMaxRows = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// acc[m] += dot(w row, x[m]) over this lane's 16-byte vectors of k (R weight rows at once;
// x's rows are ldx apart, k by default).  Each lane requests U vectors of every row
// before it multiplies any of them: 8 / R at m <= 2 (the weights are the whole cost, and
// HBM needs many bytes in flight per SM), else 4 / R (x's rows take the registers).
template <int MM, int R>
__device__ __forceinline__ void dot_rows(const uint16_t* const (&wrow)[R], const uint16_t* __restrict__ x, int k,
                                         int lane, float (&acc)[R][MM], int64_t ldx = -1) {
  constexpr int U = (MM <= 2 ? 8 : 4) / R > 0 ? (MM <= 2 ? 8 : 4) / R : 1;
  if (ldx < 0) ldx = k;
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MM; ++m) acc[r][m] = 0.f;
  const int vecs = k / 8;
  for (int v0 = lane; v0 < vecs; v0 += 32 * U) {
    uint4 a[U][R];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < R; ++r)
        a[u][r] = v0 + 32 * u < vecs ? __ldcs(reinterpret_cast<const uint4*>(wrow[r]) + v0 + 32 * u)  // streamed once
                                     : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = v0 + 32 * u;
      if (v >= vecs) break;
#pragma unroll
      for (int m = 0; m < MM; ++m) {
        const uint4 b = reinterpret_cast<const uint4*>(x + int64_t(m) * ldx)[v];
        const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a[u][r]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[r][m] = fmaf(lo_bf(pa[e]), lo_bf(pb[e]), acc[r][m]);
            acc[r][m] = fmaf(hi_bf(pa[e]), hi_bf(pb[e]), acc[r][m]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MM; ++m) acc[r][m] = warp_sum(acc[r][m]);
}

// Request the first `bytes` of a weight row towards L2 (one 128-byte line per lane and
// step): a fused-norm CTA issues this before it normalises, so its first weight batch is
// on the way while the norm's loads and reductions run.
__device__ __forceinline__ void prefetch_row_l2(const uint16_t* row, int bytes, int lane) {
  const char* p = reinterpret_cast<const char*>(row);
  for (int off = lane * 128; off < bytes; off += 32 * 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p + off));
}

// RMSNorm of the MM rows of h into shared memory (rows kNormMaxK apart), with the rounding
// of rmsnorm_kernel: y = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))), fp32 inside.  Every
// thread of the CTA takes part; each CTA of a fused projection builds its own copy (7 KB
// from L2 per row at the 7B width), which costs less than a separate launch.
constexpr int kNormMaxK = 5120;
constexpr int kNormMaxRows = 4;
template <int MM>
__device__ __forceinline__ void norm_rows(const uint16_t* __restrict__ h, const uint16_t* __restrict__ norm_w,
                                          float eps, int k, uint16_t* s_x, float* s_red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int vecs = k / 8;
  const uint4* wr = reinterpret_cast<const uint4*>(norm_w);
#pragma unroll 1
  for (int m = 0; m < MM; ++m) {
    const uint4* hr = reinterpret_cast<const uint4*>(h + int64_t(m) * k);
    float ss = 0.f;
    for (int c = threadIdx.x; c < vecs; c += blockDim.x) {
      const uint4 v = hr[c];
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float f0 = lo_bf(p[e]), f1 = hi_bf(p[e]);
        ss = __fadd_rn(ss, __fmul_rn(f0, f0));
        ss = __fadd_rn(ss, __fmul_rn(f1, f1));
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < nw; ++i) tot += s_red[i];
    const float r = rsqrtf(__fadd_rn(__fmul_rn(tot, 1.0f / float(k)), eps));
    for (int c = threadIdx.x; c < vecs; c += blockDim.x) {
      const uint4 v = hr[c], g = __ldg(wr + c);
      const uint32_t* p = reinterpret_cast<const uint32_t*>(&v);
      const uint32_t* q = reinterpret_cast<const uint32_t*>(&g);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float n0 = bf16_round(__fmul_rn(lo_bf(p[e]), r));
        const float n1 = bf16_round(__fmul_rn(hi_bf(p[e]), r));
        po[e] = pack_bf2(__fmul_rn(lo_bf(q[e]), n0), __fmul_rn(hi_bf(q[e]), n1));
      }
      *reinterpret_cast<uint4*>(s_x + int64_t(m) * kNormMaxK + c * 8) = o;
    }
    __syncthreads();  // s_red is reused by the next row; s_x complete for the dot products
  }
}

// h[m][n] = bf16(h + bf16(w[n] . x[m]))   (o_proj / down_proj + residual).  S warps share
// a row, each taking k / S of it (long rows: the down projection's 18944), and their
// partial sums meet in shared memory; a CTA of 8 warps covers 8 / S rows.
template <int MM, int S>
__global__ void __launch_bounds__(256) gemv_residual_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ w,
                                                            uint16_t* __restrict__ h, int n, int k) {
  __shared__ float s_part[8][MM];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (8 / S) + warp / S, slice = warp % S;
  const int ks = k / S;  // a multiple of 8: checked on the host
  float acc[1][MM];
  if (row < n) {
    const uint16_t* wr[1] = {w + int64_t(row) * k + int64_t(slice) * ks};
    dot_rows<MM, 1>(wr, x + int64_t(slice) * ks, ks, lane, acc, k);
  }
  if (S > 1) {
    if (lane == 0 && row < n)
#pragma unroll
      for (int m = 0; m < MM; ++m) s_part[warp][m] = acc[0][m];
    __syncthreads();
    if (row >= n || slice != 0) return;
#pragma unroll
    for (int m = 0; m < MM; ++m) {
      float t = s_part[warp][m];
#pragma unroll
      for (int q = 1; q < S; ++q) t += s_part[warp + q][m];
      acc[0][m] = t;
    }
  } else if (row >= n) {
    return;
  }
  if (lane < MM) {
    float s = acc[0][0];
#pragma unroll
    for (int m = 1; m < MM; ++m)
      if (lane == m) s = acc[0][m];
    uint16_t* hp = h + int64_t(lane) * n + row;
    *hp = f2bf(__fadd_rn(bf2f(*hp), bf16_round(s)));
  }
}

// out[m][j] = bf16(bf16(silu(bf16(g))) * bf16(u)); gate/up rows interleaved in 128-row blocks
// With kNorm, x is RMSNorm(h) with norm_w, built by the CTA (norm_rows).
template <int MM, bool kNorm>
__global__ void __launch_bounds__(256) gemv_swiglu_kernel(const uint16_t* __restrict__ x,
                                                          const uint16_t* __restrict__ w,
                                                          uint16_t* __restrict__ out, int inter, int k,
                                                          const uint16_t* __restrict__ norm_w, float eps) {
  __shared__ __align__(16) uint16_t s_x[kNorm ? MM * kNormMaxK : 8];
  __shared__ float s_red[8];
  const uint16_t* xin = x;
  int64_t ldx = k;
  const int j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int64_t gate_row = int64_t(j / 128) * 256 + (j % 128);
  const uint16_t* wr[2] = {w + gate_row * k, w + (gate_row + 128) * k};
  if constexpr (kNorm) {
    if (j < inter) {
      prefetch_row_l2(wr[0], min(k * 2, 4096), lane);
      prefetch_row_l2(wr[1], min(k * 2, 4096), lane);
    }
    norm_rows<MM>(x, norm_w, eps, k, s_x, s_red);
    xin = s_x;
    ldx = kNormMaxK;
  }
  if (j >= inter) return;
  float acc[2][MM];
  dot_rows<MM, 2>(wr, xin, k, lane, acc, ldx);
  if (lane < MM) {
    float g = acc[0][0], u = acc[1][0];
#pragma unroll
    for (int m = 1; m < MM; ++m)
      if (lane == m) {
        g = acc[0][m];
        u = acc[1][m];
      }
    const float gb = bf16_round(g);
    const float s = bf16_round(__fdiv_rn(gb, __fadd_rn(1.0f, expf(-gb))));
    out[int64_t(lane) * inter + j] = f2bf(__fmul_rn(s, bf16_round(u)));
  }
}

// q / k rows with bias and RoPE at positions[m] (a warp per rotary pair of one head: rows
// d and d + HD/2), v rows with bias; k and v go to the caches [Hk][n_ctx][HD] at pos.
template <int MM, int HD, bool kNorm>
__global__ void __launch_bounds__(256) gemv_qkv_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, const uint16_t* __restrict__ bias, int k,
    int Hq, int Hk, const int32_t* __restrict__ positions, const float2* __restrict__ rope, int rope_max_pos,
    uint16_t* __restrict__ q_out, uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache, int n_ctx,
    const uint16_t* __restrict__ norm_w, float eps) {
  constexpr int HALF = HD / 2;
  __shared__ __align__(16) uint16_t s_x[kNorm ? MM * kNormMaxK : 8];
  __shared__ float s_red[8];
  const uint16_t* xin = x;
  int64_t ldx = k;
  const int item = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int n_pair = (Hq + Hk) * HALF;
  if constexpr (kNorm) {
    if (item < n_pair) {
      const int head = item / HALF, jj = item - head * HALF;
      prefetch_row_l2(w + int64_t(head * HD + jj) * k, min(k * 2, 4096), lane);
      prefetch_row_l2(w + int64_t(head * HD + jj + HALF) * k, min(k * 2, 4096), lane);
    } else if (item < n_pair + Hk * HD) {
      prefetch_row_l2(w + int64_t((Hq + Hk) * HD + item - n_pair) * k, min(k * 2, 8192), lane);
    }
    norm_rows<MM>(x, norm_w, eps, k, s_x, s_red);
    xin = s_x;
    ldx = kNormMaxK;
  }
  if (item >= n_pair + Hk * HD) return;
  int pos = 0;
  bool ok = true;
  if (lane < MM) {
    pos = positions[lane];
    if (pos < 0 || pos >= rope_max_pos || pos >= n_ctx) {
      atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
      ok = false;
    }
  }
  if (item < n_pair) {
    const int head = item / HALF, jj = item - head * HALF;
    const int r1 = head * HD + jj, r2 = r1 + HALF;
    const uint16_t* wr[2] = {w + int64_t(r1) * k, w + int64_t(r2) * k};
    float acc[2][MM];
    dot_rows<MM, 2>(wr, xin, k, lane, acc, ldx);
    if (lane < MM && ok) {
      float d1 = acc[0][0], d2 = acc[1][0];
#pragma unroll
      for (int m = 1; m < MM; ++m)
        if (lane == m) {
          d1 = acc[0][m];
          d2 = acc[1][m];
        }
      const float a = bf16_round(__fadd_rn(d1, bf2f(bias[r1])));
      const float b = bf16_round(__fadd_rn(d2, bf2f(bias[r2])));
      const float2 cs = rope[int64_t(pos) * HALF + jj];
      const float o1 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
      const float o2 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
      uint16_t* dst = head < Hq ? q_out + (int64_t(lane) * Hq + head) * HD
                                : k_cache + (int64_t(head - Hq) * n_ctx + pos) * HD;
      dst[jj] = f2bf(o1);
      dst[jj + HALF] = f2bf(o2);
    }
  } else {
    const int vr = item - n_pair;  // v row: head vr / HD, dim vr % HD
    const int row = (Hq + Hk) * HD + vr;
    const uint16_t* wr[1] = {w + int64_t(row) * k};
    float acc[1][MM];
    dot_rows<MM, 1>(wr, xin, k, lane, acc, ldx);
    if (lane < MM && ok) {
      float d = acc[0][0];
#pragma unroll
      for (int m = 1; m < MM; ++m)
        if (lane == m) d = acc[0][m];
      v_cache[(int64_t(vr / HD) * n_ctx + pos) * HD + vr % HD] = f2bf(__fadd_rn(d, bf2f(bias[row])));
    }
  }
}

int check_gemv(const void* x, const void* w, int m, int k, const char* name) {
  CKV_REQUIRE(x && w, "%s: null pointer", name);
  CKV_REQUIRE(m >= 1 && m <= kMaxRows, "%s: m=%d outside 1..%d", name, m, kMaxRows);
  CKV_REQUIRE(k > 0 && k % 8 == 0 && aligned16(x) && aligned16(w), "%s: k %% 8 and 16-byte alignment", name);
  return CKV_OK;
}

}  // namespace
}  // namespace ckv

using namespace ckv;

// x rows, or (norm_w != nullptr) the rows of h to RMSNorm first: at most kNormMaxRows rows
// of at most kNormMaxK columns, the CTA's copy in shared memory
static int check_norm(const uint16_t* norm_w, int m, int k, const char* name) {
  if (norm_w == nullptr) return CKV_OK;
  CKV_REQUIRE(aligned16(norm_w), "%s: norm weight must be 16-byte aligned", name);
  CKV_REQUIRE(m <= kNormMaxRows && k <= kNormMaxK, "%s: m=%d, k=%d beyond the fused norm's %d x %d", name, m, k,
              kNormMaxRows, kNormMaxK);
  return CKV_OK;
}

#define CKV_NORM_SWITCH(m, LAUNCH, NORM) \
  switch (m) {                           \
    case 1: LAUNCH(1, NORM); break;      \
    case 2: LAUNCH(2, NORM); break;      \
    case 3: LAUNCH(3, NORM); break;      \
    case 4: LAUNCH(4, NORM); break;      \
    case 5: LAUNCH(5, NORM); break;      \
    case 6: LAUNCH(6, NORM); break;      \
    case 7: LAUNCH(7, NORM); break;      \
    default: LAUNCH(8, NORM); break;     \
  }
#define CKV_NORM_SWITCH4(m, LAUNCH) \
  switch (m) {                      \
    case 1: LAUNCH(1, true); break; \
    case 2: LAUNCH(2, true); break; \
    case 3: LAUNCH(3, true); break; \
    default: LAUNCH(4, true); break; \
  }

static int gemv_swiglu_launch(const uint16_t* x, const uint16_t* norm_w, float eps, const uint16_t* w_gate_up,
                              uint16_t* out, int m, int inter, int k, ckv_stream_t stream, const char* name) {
  if (int rc = check_gemv(x, w_gate_up, m, k, name)) return rc;
  if (int rc = check_norm(norm_w, m, k, name)) return rc;
  CKV_REQUIRE(out && inter > 0 && inter % 128 == 0, "%s: inter %d not a multiple of 128", name, inter);
  const int grid = ceil_div(inter, 8);
  cudaStream_t s = as_stream(stream);
#define CKV_L(MM, NORM) gemv_swiglu_kernel<MM, NORM><<<grid, 256, 0, s>>>(x, w_gate_up, out, inter, k, norm_w, eps)
  if (norm_w) {
    CKV_NORM_SWITCH4(m, CKV_L)
  } else {
    CKV_NORM_SWITCH(m, CKV_L, false)
  }
#undef CKV_L
  CKV_LAUNCH_CHECK(name);
  return CKV_OK;
}

static int gemv_qkv_launch(const uint16_t* x, const uint16_t* norm_w, float eps, const uint16_t* w_qkv,
                           const uint16_t* b_qkv, int m, int k, int n_q_heads, int n_kv_heads, int head_dim,
                           const int32_t* positions, const float* rope_table, int rope_max_pos, uint16_t* q_out,
                           uint16_t* k_cache, uint16_t* v_cache, int n_ctx, ckv_stream_t stream, const char* name) {
  if (int rc = check_gemv(x, w_qkv, m, k, name)) return rc;
  if (int rc = check_norm(norm_w, m, k, name)) return rc;
  CKV_REQUIRE(b_qkv && positions && rope_table && q_out && k_cache && v_cache, "%s: null pointer", name);
  CKV_REQUIRE(n_q_heads > 0 && n_kv_heads > 0 && n_ctx > 0 && rope_max_pos > 0, "%s: bad sizes", name);
  const int items = (n_q_heads + n_kv_heads) * (head_dim / 2) + n_kv_heads * head_dim;
  const int grid = ceil_div(items, 8);
  cudaStream_t s = as_stream(stream);
  const float2* rope = reinterpret_cast<const float2*>(rope_table);
  if (head_dim == 128) {
#define CKV_L(MM, NORM)                                                                                        \
  gemv_qkv_kernel<MM, 128, NORM><<<grid, 256, 0, s>>>(x, w_qkv, b_qkv, k, n_q_heads, n_kv_heads, positions,    \
                                                      rope, rope_max_pos, q_out, k_cache, v_cache, n_ctx, norm_w, \
                                                      eps)
    if (norm_w) {
      CKV_NORM_SWITCH4(m, CKV_L)
    } else {
      CKV_NORM_SWITCH(m, CKV_L, false)
    }
#undef CKV_L
  } else if (head_dim == 64) {
#define CKV_L(MM, NORM)                                                                                       \
  gemv_qkv_kernel<MM, 64, NORM><<<grid, 256, 0, s>>>(x, w_qkv, b_qkv, k, n_q_heads, n_kv_heads, positions,    \
                                                     rope, rope_max_pos, q_out, k_cache, v_cache, n_ctx, norm_w, \
                                                     eps)
    if (norm_w) {
      CKV_NORM_SWITCH4(m, CKV_L)
    } else {
      CKV_NORM_SWITCH(m, CKV_L, false)
    }
#undef CKV_L
  } else {
    set_error("%s: head_dim %d (64 or 128)", name, head_dim);
    return CKV_ERR_UNSUPPORTED;
  }
  CKV_LAUNCH_CHECK(name);
  return CKV_OK;
}

#define CKV_GEMV_SWITCH(m, LAUNCH) \
  switch (m) {                     \
    case 1: LAUNCH(1); break;      \
    case 2: LAUNCH(2); break;      \
    case 3: LAUNCH(3); break;      \
    case 4: LAUNCH(4); break;      \
    case 5: LAUNCH(5); break;      \
    case 6: LAUNCH(6); break;      \
    case 7: LAUNCH(7); break;      \
    default: LAUNCH(8); break;     \
  }

extern "C" {

int ckv_gemv_residual(const uint16_t* x, const uint16_t* w, uint16_t* h, int m, int n, int k,
                      ckv_stream_t stream) {
  if (int rc = check_gemv(x, w, m, k, "ckv_gemv_residual")) return rc;
  CKV_REQUIRE(h, "ckv_gemv_residual: null h");
  if (n <= 0) return CKV_OK;
  cudaStream_t s = as_stream(stream);
  if (k >= 8192 && k % 32 == 0) {  // long rows: four warps per row
    const int grid = ceil_div(n, 2);
#define CKV_L(MM) gemv_residual_kernel<MM, 4><<<grid, 256, 0, s>>>(x, w, h, n, k)
    CKV_GEMV_SWITCH(m, CKV_L)
#undef CKV_L
  } else {
    const int grid = ceil_div(n, 8);
#define CKV_L(MM) gemv_residual_kernel<MM, 1><<<grid, 256, 0, s>>>(x, w, h, n, k)
    CKV_GEMV_SWITCH(m, CKV_L)
#undef CKV_L
  }
  CKV_LAUNCH_CHECK("ckv_gemv_residual");
  return CKV_OK;
}

int ckv_gemv_swiglu(const uint16_t* x, const uint16_t* w_gate_up, uint16_t* out, int m, int inter, int k,
                    ckv_stream_t stream) {
  return gemv_swiglu_launch(x, nullptr, 0.f, w_gate_up, out, m, inter, k, stream, "ckv_gemv_swiglu");
}

int ckv_gemv_swiglu_rmsnorm(const uint16_t* h, const uint16_t* norm_w, float eps, const uint16_t* w_gate_up,
                            uint16_t* out, int m, int inter, int k, ckv_stream_t stream) {
  CKV_REQUIRE(norm_w, "ckv_gemv_swiglu_rmsnorm: null norm weight");
  return gemv_swiglu_launch(h, norm_w, eps, w_gate_up, out, m, inter, k, stream, "ckv_gemv_swiglu_rmsnorm");
}

int ckv_gemv_qkv_rope(const uint16_t* x, const uint16_t* w_qkv, const uint16_t* b_qkv, int m, int k,
                      int n_q_heads, int n_kv_heads, int head_dim, const int32_t* positions,
                      const float* rope_table, int rope_max_pos, uint16_t* q_out, uint16_t* k_cache,
                      uint16_t* v_cache, int n_ctx, ckv_stream_t stream) {
  return gemv_qkv_launch(x, nullptr, 0.f, w_qkv, b_qkv, m, k, n_q_heads, n_kv_heads, head_dim, positions,
                         rope_table, rope_max_pos, q_out, k_cache, v_cache, n_ctx, stream, "ckv_gemv_qkv_rope");
}

int ckv_gemv_qkv_rope_rmsnorm(const uint16_t* h, const uint16_t* norm_w, float eps, const uint16_t* w_qkv,
                              const uint16_t* b_qkv, int m, int k, int n_q_heads, int n_kv_heads, int head_dim,
                              const int32_t* positions, const float* rope_table, int rope_max_pos,
                              uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, int n_ctx,
                              ckv_stream_t stream) {
  CKV_REQUIRE(norm_w, "ckv_gemv_qkv_rope_rmsnorm: null norm weight");
  return gemv_qkv_launch(h, norm_w, eps, w_qkv, b_qkv, m, k, n_q_heads, n_kv_heads, head_dim, positions,
                         rope_table, rope_max_pos, q_out, k_cache, v_cache, n_ctx, stream,
                         "ckv_gemv_qkv_rope_rmsnorm");
}

}  // extern "C"
