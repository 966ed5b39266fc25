// Attention of the recomputed tokens over the blended cache (torch_engine.py:68-70,157).
//
// Query row i (a token at absolute position positions[i]) sees key j iff
// j <= positions[i]; the cache holds every position 0..n_ctx-1 (moved cached
// K/V plus freshly written rows).  GQA: the G = Hq/Hk query heads that share a
// KV head are packed as consecutive rows (row = token*G + g), so one K/V tile
// serves G heads.  Flash-style: online softmax in fp32 (exp2 with the scale
// folded in), P rounded to bf16 for the P.V product, output divided by the
// row sum at the end.  Tensor-core path: mma.sync m16n8k16 bf16 (ldmatrix
// operands from XOR-swizzled shared memory), K/V tiles double-buffered with
// cp.async.  CTA = 4 warps x 16 rows; key tiles of 64.
#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(attention)

namespace ckv {
namespace {

constexpr int BR = 64;  // packed query rows per CTA
constexpr int BC = 64;  // keys per tile
constexpr int kThreads = 128;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0 -> zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                      uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2(float a, float b) { return pack_bf2(a, b); }

// element offset of (row, 16-byte chunk) in a [rows][HD] tile, chunk XOR-swizzled by row
template <int HD>
__device__ __forceinline__ int swz(int r, int ch) {
  return r * HD + ((ch ^ (r & 7)) << 3);
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 2)
    attention_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kc,
                     const uint16_t* __restrict__ vc, const int32_t* __restrict__ positions,
                     uint16_t* __restrict__ out, int M, int Hq, int Hk, int n_ctx,
                     float scale_log2) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint16_t smem[];
  uint16_t* sQ = smem;                  // [BR][HD]
  uint16_t* sK = sQ + BR * HD;          // [2][BC][HD]
  uint16_t* sV = sK + 2 * BC * HD;      // [2][BC][HD]
  __shared__ int s_minmax[2];

  const int G = Hq / Hk;
  const int hk = blockIdx.y;
  const int rb = gridDim.x - 1 - blockIdx.x;  // heavy (late-position) blocks first
  const int R = M * G;
  const int R0 = rb * BR;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // key range of this block: positions of its first / last token (any order tolerated)
  if (tid == 0) {
    s_minmax[0] = 0x7fffffff;
    s_minmax[1] = -1;
  }
  __syncthreads();
  {
    const int t_first = R0 / G, t_last = min(R0 + BR, R) - 1;
    for (int t = t_first + tid; t <= t_last / G; t += kThreads) {
      int p = positions[t];
      if (p < 0 || p >= n_ctx) {
        atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
        p = p < 0 ? 0 : n_ctx - 1;
      }
      atomicMin(&s_minmax[0], p);
      atomicMax(&s_minmax[1], p);
    }
  }
  __syncthreads();
  const int min_pos = s_minmax[0], max_pos = s_minmax[1];
  const int n_kt = (max_pos + 1 + BC - 1) / BC;

  const uint16_t* kbase = kc + int64_t(hk) * n_ctx * HD;
  const uint16_t* vbase = vc + int64_t(hk) * n_ctx * HD;

  // Q tile
  for (int i = tid; i < BR * CH; i += kThreads) {
    const int r = i / CH, ch = i - r * CH;
    const int gr = R0 + r;
    const bool valid = gr < R;
    const int t = valid ? gr / G : 0, g = valid ? gr - (gr / G) * G : 0;
    const uint16_t* src = q + (int64_t(t) * Hq + hk * G + g) * HD + ch * 8;
    cp_async16(smem_u32(sQ + swz<HD>(r, ch)), valid ? src : q, valid);
  }
  auto load_kv = [&](int kt, int buf) {
    const int j0 = kt * BC;
    for (int i = tid; i < BC * CH; i += kThreads) {
      const int r = i / CH, ch = i - r * CH;
      const int j = j0 + r;
      // keys past the block's last position are never visible: zero them instead of
      // reading rows the caller may not have written (0 * garbage could be NaN)
      const bool valid = j <= max_pos;
      const int64_t off = int64_t(valid ? j : 0) * HD + ch * 8;
      cp_async16(smem_u32(sK + buf * BC * HD + swz<HD>(r, ch)), kbase + off, valid);
      cp_async16(smem_u32(sV + buf * BC * HD + swz<HD>(r, ch)), vbase + off, valid);
    }
  };
  if (n_kt > 0) load_kv(0, 0);
  cp_commit();

  // rows owned by this thread: r_a = 16*warp + lane/4 and r_a + 8
  const int ra = warp * 16 + (lane >> 2);
  int pos_a = 0, pos_b = 0;
  {
    const int ga = R0 + ra, gb = R0 + ra + 8;
    if (ga < R) pos_a = min(max(positions[ga / G], 0), n_ctx - 1);
    if (gb < R) pos_b = min(max(positions[gb / G], 0), n_ctx - 1);
  }

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  uint32_t qf[HD / 16][4];

  for (int kt = 0; kt < n_kt; ++kt) {
    if (kt + 1 < n_kt) load_kv(kt + 1, (kt + 1) & 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = ks * 2 + (lane >> 4);
        ldsm4(smem_u32(sQ + swz<HD>(r, ch)), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
      }
    }
    const uint16_t* cK = sK + (kt & 1) * BC * HD;
    const uint16_t* cV = sV + (kt & 1) * BC * HD;

    // S = Q K^T (16 rows x 64 keys per warp)
    float s[BC / 8][4];
#pragma unroll
    for (int i = 0; i < BC / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < BC / 16; ++np) {
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int ch = ks * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm4(smem_u32(cK + swz<HD>(r, ch)), b0, b1, b2, b3);
        mma16816(s[2 * np], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
        mma16816(s[2 * np + 1], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b2, b3);
      }
    }
    // mask keys past each row's position
    const int j0 = kt * BC;
    if (j0 + BC - 1 > min_pos) {
#pragma unroll
      for (int nt = 0; nt < BC / 8; ++nt) {
        const int j = j0 + nt * 8 + 2 * (lane & 3);
        if (j > pos_a) s[nt][0] = -INFINITY;
        if (j + 1 > pos_a) s[nt][1] = -INFINITY;
        if (j > pos_b) s[nt][2] = -INFINITY;
        if (j + 1 > pos_b) s[nt][3] = -INFINITY;
      }
    }
    // online softmax
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < BC / 8; ++nt) {
      mx_a = fmaxf(mx_a, fmaxf(s[nt][0], s[nt][1]));
      mx_b = fmaxf(mx_b, fmaxf(s[nt][2], s[nt][3]));
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
    }
    const float mn_a = fmaxf(m_a, mx_a * scale_log2);
    const float mn_b = fmaxf(m_b, mx_b * scale_log2);
    const float base_a = mn_a == -INFINITY ? 0.f : mn_a;
    const float base_b = mn_b == -INFINITY ? 0.f : mn_b;
    const float corr_a = exp2f(m_a - base_a), corr_b = exp2f(m_b - base_b);
    m_a = mn_a;
    m_b = mn_b;
    float rs_a = 0.f, rs_b = 0.f;
#pragma unroll
    for (int nt = 0; nt < BC / 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] * scale_log2 - base_a);
      s[nt][1] = exp2f(s[nt][1] * scale_log2 - base_a);
      s[nt][2] = exp2f(s[nt][2] * scale_log2 - base_b);
      s[nt][3] = exp2f(s[nt][3] * scale_log2 - base_b);
      rs_a += s[nt][0] + s[nt][1];
      rs_b += s[nt][2] + s[nt][3];
    }
    l_a = l_a * corr_a + rs_a;
    l_b = l_b * corr_b + rs_b;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= corr_a;
      o[i][1] *= corr_a;
      o[i][2] *= corr_b;
      o[i][3] *= corr_b;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BC / 16; ++kk) {
      const uint32_t a0 = pack2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = dp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm4_t(smem_u32(cV + swz<HD>(r, ch)), b0, b1, b2, b3);
        mma16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // this buffer is refilled two iterations later
  }
  cp_wait<0>();

  // row sums across the 4 lanes of a row, normalise, stage through sQ, store
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
  }
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f;
  const float inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  __syncthreads();
#pragma unroll
  for (int nd = 0; nd < HD / 8; ++nd) {
    const int c = nd * 8 + 2 * (lane & 3);
    uint32_t* pa = reinterpret_cast<uint32_t*>(sQ + swz<HD>(ra, c >> 3) + (c & 7));
    uint32_t* pb = reinterpret_cast<uint32_t*>(sQ + swz<HD>(ra + 8, c >> 3) + (c & 7));
    *pa = pack2(o[nd][0] * inv_a, o[nd][1] * inv_a);
    *pb = pack2(o[nd][2] * inv_b, o[nd][3] * inv_b);
  }
  __syncthreads();
  for (int i = tid; i < BR * CH; i += kThreads) {
    const int r = i / CH, ch = i - r * CH;
    const int gr = R0 + r;
    if (gr >= R) continue;
    const int t = gr / G, g = gr - t * G;
    uint16_t* dst = out + (int64_t(t) * Hq + hk * G + g) * HD + ch * 8;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(sQ + swz<HD>(r, ch));
  }
}

template <int HD>
int launch(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* positions,
           uint16_t* out, int M, int Hq, int Hk, int n_ctx, float scale, cudaStream_t stream) {
  const int smem = (BR + 4 * BC) * HD * 2;
  auto kern = attention_kernel<HD>;
  if (int rc = set_smem_limit(reinterpret_cast<const void*>(kern), smem)) return rc;
  const int G = Hq / Hk;
  const int64_t rows = int64_t(M) * G;
  const int blocks = ceil_div(rows, BR);
  kern<<<dim3(blocks, Hk), kThreads, smem, stream>>>(q, kc, vc, positions, out, M, Hq, Hk, n_ctx,
                                                     scale * 1.4426950408889634f);
  CKV_LAUNCH_CHECK("ckv_attention");
  return CKV_OK;
}

}  // namespace
}  // namespace ckv

using namespace ckv;

extern "C" {

int ckv_attention(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                  const int32_t* positions, uint16_t* out, int m, int n_q_heads, int n_kv_heads,
                  int head_dim, int n_ctx, float scale, ckv_stream_t stream) {
  CKV_REQUIRE(q && k_cache && v_cache && positions && out, "ckv_attention: null pointer");
  CKV_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out),
              "ckv_attention: tensors must be 16-byte aligned");
  CKV_REQUIRE(n_kv_heads > 0 && n_q_heads % n_kv_heads == 0,
              "ckv_attention: n_q_heads %d not a multiple of n_kv_heads %d", n_q_heads, n_kv_heads);
  CKV_REQUIRE(n_kv_heads <= 65535 && n_ctx > 0 && m >= 0, "ckv_attention: bad sizes");
  if (m == 0) return CKV_OK;
  if (head_dim == 128)
    return launch<128>(q, k_cache, v_cache, positions, out, m, n_q_heads, n_kv_heads, n_ctx, scale,
                       as_stream(stream));
  if (head_dim == 64)
    return launch<64>(q, k_cache, v_cache, positions, out, m, n_q_heads, n_kv_heads, n_ctx, scale,
                      as_stream(stream));
  set_error("ckv_attention: head_dim %d (64 or 128)", head_dim);
  return CKV_ERR_UNSUPPORTED;
}

}  // extern "C"
