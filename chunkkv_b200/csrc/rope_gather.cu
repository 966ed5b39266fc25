// Re-RoPE and the store <-> blended-cache copies (HBM-streaming kernels).
//
// Rotation arithmetic follows TorchEngine._rotate (torch_engine.py:46-51):
// angle = fp32(delta * inv_freq[j]); out1 = x1*cos - x2*sin, out2 = x1*sin + x2*cos,
// each product and sum rounded in fp32 (no FMA contraction), result rounded to
// bf16.  Pairs are (j, j + rot/2) for j < rot/2 (half-split layout,
// rerope.py:36-47); dims >= rot are copied unchanged.
//
// Work unit of the gather/scatter kernels: 16 tokens (one page block) of one
// (layer, K|V, kv-head) — 16 * head_dim * 2 bytes, contiguous on both sides.
#include "ckv_common.cuh"

CKV_DEFINE_ERR_WORD(rope)

namespace ckv {
namespace {

constexpr int kPage = CKV_PAGE_TOKENS;
constexpr int kMaxHalf = 128;  // rot_dims <= 256
constexpr int kSmemPages = 1024;  // page ids of a chunk kept in shared memory (16k tokens)
constexpr int kCopyWarps = 8;     // warps of a 256-thread copy CTA
constexpr int kStageVec = 256;    // 16-byte vectors in a warp's staging slot (4 KiB)

struct uint4x2 {
  uint4 a, b;
};

// Rotate 8 (x1, x2) pairs held as two 16-byte vectors.
__device__ __forceinline__ void rotate8(uint4& v1, uint4& v2, const float2* cs) {
  uint32_t* p1 = reinterpret_cast<uint32_t*>(&v1);
  uint32_t* p2 = reinterpret_cast<uint32_t*>(&v2);
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    float a[2] = {lo_bf(p1[w]), hi_bf(p1[w])};
    float b[2] = {lo_bf(p2[w]), hi_bf(p2[w])};
    float o1[2], o2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float c = cs[2 * w + e].x, s = cs[2 * w + e].y;
      o1[e] = __fsub_rn(__fmul_rn(a[e], c), __fmul_rn(b[e], s));
      o2[e] = __fadd_rn(__fmul_rn(a[e], s), __fmul_rn(b[e], c));
    }
    p1[w] = pack_bf2(o1[0], o1[1]);
    p2[w] = pack_bf2(o2[0], o2[1]);
  }
}

__device__ __forceinline__ float2 rope_cs(float pos_or_delta, float inv_freq) {
  const float a = __fmul_rn(pos_or_delta, inv_freq);
  return make_float2(cosf(a), sinf(a));
}

// n_vec contiguous 16-byte vectors from src to dst by one warp, through the warp's 4 KiB
// shared staging slot: cp.async puts a whole slot of loads in flight (a 16-token page plane
// at head_dim 128 in one round trip) without holding them in registers.  Each lane stores
// only the vectors it copied itself, so its own wait_group is the only ordering needed.
__device__ __forceinline__ void copy_flat_warp(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                               int n_vec, uint4* stage, int lane) {
  const unsigned stage_s = static_cast<unsigned>(__cvta_generic_to_shared(stage));
  for (int i0 = 0; i0 < n_vec; i0 += kStageVec) {
    const int n = min(kStageVec, n_vec - i0);
    __syncwarp();  // the slot's previous contents have been read by every lane
    for (int i = lane; i < n; i += 32)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(stage_s + 16u * i), "l"(src + i0 + i)
                   : "memory");
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    for (int i = lane; i < n; i += 32) __stcs(dst + i0 + i, stage[i]);
  }
}

// `rows` rows of head_dim bf16, contiguous on both sides, rotated by the per-j table cs
// (smem).  The rows come into the warp's staging slot by cp.async (a 16-row slice at
// head_dim 128 in one fill, every load in flight, none held in registers); then each lane
// takes rotary pairs (vectors p and p + rot/16 of a row) and the unrotated vectors past
// rot out of shared memory and stores them.
__device__ __forceinline__ void rotate_rows_staged_warp(const uint16_t* __restrict__ src,
                                                        uint16_t* __restrict__ dst, int rows, int head_dim,
                                                        int rot, const float2* cs, uint4* stage, int lane) {
  const int vec_row = head_dim / 8;               // 16-byte vectors per row
  const int rows_per_fill = kStageVec / vec_row;  // >= 8: head_dim <= 256
  const int n_pair = rot / 16;                    // partner vector of p is p + n_pair
  const int per_row = vec_row - n_pair;           // pair items + unrotated vectors
  const unsigned stage_s = static_cast<unsigned>(__cvta_generic_to_shared(stage));
  for (int r0 = 0; r0 < rows; r0 += rows_per_fill) {
    const int nr = min(rows_per_fill, rows - r0);
    const uint4* s4 = reinterpret_cast<const uint4*>(src + int64_t(r0) * head_dim);
    uint4* d4 = reinterpret_cast<uint4*>(dst + int64_t(r0) * head_dim);
    __syncwarp();  // every lane has read the slot's previous contents
    for (int i = lane; i < nr * vec_row; i += 32)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(stage_s + 16u * i), "l"(s4 + i) : "memory");
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncwarp();  // every lane's copies have landed: lanes read each other's vectors below
    for (int it = lane; it < nr * per_row; it += 32) {
      const int r = it / per_row, item = it - r * per_row;
      const int base = r * vec_row;
      if (item < n_pair) {
        uint4 v1 = stage[base + item], v2 = stage[base + item + n_pair];
        rotate8(v1, v2, cs + item * 8);
        __stcs(d4 + base + item, v1);
        __stcs(d4 + base + item + n_pair, v2);
      } else {
        const int v = item + n_pair;  // vectors 2 * n_pair .. vec_row - 1
        __stcs(d4 + base + v, stage[base + v]);
      }
    }
  }
}

__global__ void rope_table_kernel(const float* __restrict__ inv_freq, int half, int max_pos,
                                  float2* __restrict__ table) {
  const int64_t n = int64_t(max_pos) * half;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int p = int(i / half), j = int(i - int64_t(p) * half);
    table[i] = rope_cs(float(p), inv_freq[j]);
  }
}

// dst[row] = rotate(src[row], cs(delta)) for every row: the (cos, sin) of the one angle per
// rotary pair are computed once per CTA into shared memory; warps copy 16-row units
// (4 KiB at head_dim 128) through each warp's shared staging slot.
__global__ void __launch_bounds__(256, 4) shift_rows_kernel(const uint16_t* __restrict__ src,
                                                         uint16_t* __restrict__ dst, int64_t rows,
                                                         int head_dim, int rot, int delta,
                                                         const float* __restrict__ inv_freq) {
  __shared__ float2 cs[kMaxHalf];
  __shared__ __align__(16) uint4 s_stage[kCopyWarps][kStageVec];
  pdl_wait();  // the rows come from the kernel before (dependent launch)
  pdl_launch_next();
  for (int j = threadIdx.x; j < rot / 2; j += blockDim.x) cs[j] = rope_cs(float(delta), inv_freq[j]);
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t n_units = (rows + kPage - 1) / kPage;
  for (int64_t u = int64_t(blockIdx.x) * 8 + warp; u < n_units; u += int64_t(gridDim.x) * 8) {
    const int64_t r0 = u * kPage;
    const int n = int(min(int64_t(kPage), rows - r0));
    rotate_rows_staged_warp(src + r0 * head_dim, dst + r0 * head_dim, n, head_dim, rot, cs, s_stage[warp], lane);
  }
}

// dst[row] = rotate(src[row], cs(pos(row))) with pos = delta (shift) or positions[row % seq].
__global__ void rope_rows_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                                 int64_t rows, int head_dim, int rot, int delta,
                                 const int32_t* __restrict__ positions, int seq,
                                 const float* __restrict__ inv_freq) {
  const int n_pair = rot / 16;
  const int n_copy = head_dim / 8 - 2 * n_pair;
  const int per_row = n_pair + n_copy;
  const int64_t total = rows * per_row;
  for (int64_t it = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; it < total;
       it += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = it / per_row;
    const int item = int(it - r * per_row);
    const uint16_t* s = src + r * head_dim;
    uint16_t* d = dst + r * head_dim;
    if (item < n_pair) {
      const int j = item * 8;
      const float p = positions ? float(positions[r % seq]) : float(delta);
      float2 cs[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) cs[e] = rope_cs(p, inv_freq[j + e]);
      uint4 v1 = *reinterpret_cast<const uint4*>(s + j);
      uint4 v2 = *reinterpret_cast<const uint4*>(s + j + rot / 2);
      rotate8(v1, v2, cs);
      *reinterpret_cast<uint4*>(d + j) = v1;
      *reinterpret_cast<uint4*>(d + j + rot / 2) = v2;
    } else {
      const int off = rot + (item - n_pair) * 8;
      *reinterpret_cast<uint4*>(d + off) = *reinterpret_cast<const uint4*>(s + off);
    }
  }
}

// fp32 rows (torch_engine.py:46-51 with x.dtype float32: the result stays fp32):
// dst[row] = rotate(src[row], cs(pos(row))), four rotary pairs per item as two float4,
// pos = delta (shift) or positions[row % seq]; dims past rot copied.
__global__ void rope_rows_f32_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t rows,
                                     int head_dim, int rot, int delta, const int32_t* __restrict__ positions,
                                     int seq, const float* __restrict__ inv_freq) {
  const int n_pair = rot / 8;
  const int n_copy = (head_dim - rot) / 4;
  const int per_row = n_pair + n_copy;
  const int64_t total = rows * per_row;
  for (int64_t it = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; it < total;
       it += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = it / per_row;
    const int item = int(it - r * per_row);
    const float* s = src + r * head_dim;
    float* d = dst + r * head_dim;
    if (item < n_pair) {
      const int j = item * 4;
      const float p = positions ? float(positions[r % seq]) : float(delta);
      const float4 a4 = *reinterpret_cast<const float4*>(s + j);
      const float4 b4 = *reinterpret_cast<const float4*>(s + j + rot / 2);
      const float a[4] = {a4.x, a4.y, a4.z, a4.w}, b[4] = {b4.x, b4.y, b4.z, b4.w};
      float o1[4], o2[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 cs = rope_cs(p, inv_freq[j + e]);
        o1[e] = __fsub_rn(__fmul_rn(a[e], cs.x), __fmul_rn(b[e], cs.y));
        o2[e] = __fadd_rn(__fmul_rn(a[e], cs.y), __fmul_rn(b[e], cs.x));
      }
      *reinterpret_cast<float4*>(d + j) = make_float4(o1[0], o1[1], o1[2], o1[3]);
      *reinterpret_cast<float4*>(d + j + rot / 2) = make_float4(o2[0], o2[1], o2[2], o2[3]);
    } else {
      const int off = rot + (item - n_pair) * 4;
      *reinterpret_cast<float4*>(d + off) = *reinterpret_cast<const float4*>(s + off);
    }
  }
}

int launch_rope_f32(const float* src, float* dst, int64_t rows, int head_dim, int rot, int delta,
                    const int32_t* positions, int seq, const float* inv_freq, cudaStream_t st,
                    const char* name) {
  const int64_t items = rows * (rot / 8 + (head_dim - rot) / 4);
  const int grid = static_cast<int>(std::min<int64_t>((items + 255) / 256, 16 * num_sms()));
  rope_rows_f32_kernel<<<grid, 256, 0, st>>>(src, dst, rows, head_dim, rot, delta, positions, seq, inv_freq);
  CKV_LAUNCH_CHECK(name);
  return CKV_OK;
}

// One CTA column (blockIdx.y) per chunk; warps stride over the chunk's units.
// Unit u -> (block b, head h, kv, layer l), block fastest so consecutive warps write
// consecutive 4 KiB pieces of the same (layer, K|V, head) plane of the blended cache
// (measured 4 % faster than reading consecutive pieces of one page).  Stores stream
// (evict-first): the cache is read back layer by layer, long after this kernel.
template <bool kPaged>
__global__ void __launch_bounds__(256, 4) blend_gather_kernel(
    const uint16_t* __restrict__ pool, int64_t n_pages, const int32_t* __restrict__ page_table,
    const uint64_t* __restrict__ k_ptrs, const uint64_t* __restrict__ v_ptrs,
    const int32_t* __restrict__ chunk_meta, const float* __restrict__ inv_freq, int rot,
    uint16_t* __restrict__ k_out, uint16_t* __restrict__ v_out, int layer_lo, int layer_hi,
    int n_layers, int H, int D, int n_ctx) {
  __shared__ float2 cs[kMaxHalf];
  __shared__ int s_pages[kSmemPages];  // this chunk's page ids, so no unit waits on a table load
  __shared__ __align__(16) uint4 s_stage[kCopyWarps][kStageVec];  // plain (V, Δ = 0) units
  pdl_wait();  // the chunk tables and pages come from the work before (dependent launch)
  pdl_launch_next();
  const int32_t* meta = chunk_meta + blockIdx.y * CKV_META_STRIDE;
  const int table_off = meta[CKV_META_TABLE_OFFSET];
  const int length = meta[CKV_META_LENGTH];
  const int dst_start = meta[CKV_META_DST_START];
  const int delta = meta[CKV_META_DELTA];
  const int lb = max(layer_lo, meta[CKV_META_LAYER_BEGIN]);
  const int le = min(layer_hi, meta[CKV_META_LAYER_END]);
  const int src_off = meta[CKV_META_SRC_OFFSET];
  const int64_t head_stride = meta[CKV_META_HEAD_STRIDE];
  if (le <= lb || length <= 0) return;
  const bool rotate = delta != 0;
  if (rotate)
    for (int j = threadIdx.x; j < rot / 2; j += blockDim.x) cs[j] = rope_cs(float(delta), inv_freq[j]);
  const int n_slots = kPaged ? min(kSmemPages, (src_off + length + kPage - 1) / kPage) : 0;
  for (int i = threadIdx.x; i < n_slots; i += blockDim.x) s_pages[i] = page_table[table_off + i];
  __syncthreads();

  const int nl = le - lb;
  const int n_blocks = (length + kPage - 1) / kPage;
  const int n_units = n_blocks * nl * 2 * H;  // < 2^31: checked on the host
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int warps = blockDim.x / 32;
  const int64_t layer_elems = int64_t(H) * n_ctx * D;
  for (int u = blockIdx.x * warps + warp; u < n_units; u += gridDim.x * warps) {
    int t = u;
    const int b = t % n_blocks;
    t /= n_blocks;
    const int h = t % H;
    t /= H;
    const int kv = t & 1;
    t >>= 1;
    const int l = lb + t;
    const int r0 = b * kPage;
    const int rows = min(kPage, length - r0);
    const int dpos = dst_start + r0;
    if (dpos < 0 || dpos + rows > n_ctx) {
      if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
      continue;
    }
    uint16_t* dst = (kv ? v_out : k_out) + int64_t(l - layer_lo) * layer_elems +
                    (int64_t(h) * n_ctx + dpos) * D;
    const bool rot_this = rotate && kv == 0;
    if (kPaged) {
      // rows may straddle two pages when src_off is not page aligned: split
      int done = 0;
      while (done < rows) {
        const int tok = src_off + r0 + done;
        const int slot = tok / kPage, in_page = tok % kPage;
        const int take = min(rows - done, kPage - in_page);
        const int page = slot < kSmemPages ? s_pages[slot] : page_table[table_off + slot];
        if (page < 0 || page >= n_pages) {
          if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_PAGE_RANGE);
        } else {
          const uint16_t* src = pool + ((((int64_t(page) * n_layers + l) * 2 + kv) * H + h) * kPage + in_page) * D;
          if (rot_this)
            rotate_rows_staged_warp(src, dst + int64_t(done) * D, take, D, rot, cs, s_stage[warp], lane);
          else
            copy_flat_warp(reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst + int64_t(done) * D),
                           take * (D / 8), s_stage[warp], lane);
        }
        done += take;
      }
    } else {
      const uint64_t base = (kv ? v_ptrs : k_ptrs)[table_off + l];
      if ((base & 15u) != 0 || (head_stride & 7) != 0) {  // would break 16-byte vector loads
        if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
        continue;
      }
      const uint16_t* src = reinterpret_cast<const uint16_t*>(base) + h * head_stride +
                            int64_t(src_off + r0) * D;
      if (rot_this)
        rotate_rows_staged_warp(src, dst, rows, D, rot, cs, s_stage[warp], lane);
      else
        copy_flat_warp(reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), rows * (D / 8),
                       s_stage[warp], lane);
    }
  }
}

// Paged gather through a ring of TMA bulk copies.  A warp takes the same units as
// blend_gather_kernel (16 tokens of one (layer, K|V, head), one or two page pieces) and
// keeps kRing of them in its own shared-memory slots: its lane 0 loads unit k + kRing - 1
// (cp.async.bulk from the page pool, completing on the slot's mbarrier) while unit k is
// stored.  A plain unit (V, or K with delta = 0) goes back out by one bulk store from the
// slot, so its bytes never pass through registers; a unit to re-rope is rotated in place
// in the slot by the warp's lanes (the same fp32 rotation as rotate8) and then stored the
// same way.  Every wait is bounded.
constexpr int kRing = 3;
__global__ void __launch_bounds__(256, 2) blend_gather_bulk_kernel(
    const uint16_t* __restrict__ pool, int64_t n_pages, const int32_t* __restrict__ page_table,
    const int32_t* __restrict__ chunk_meta, const float* __restrict__ inv_freq, int rot,
    uint16_t* __restrict__ k_out, uint16_t* __restrict__ v_out, int layer_lo, int layer_hi, int n_layers,
    int H, int D, int n_ctx) {
  extern __shared__ __align__(128) uint8_t ring_raw[];
  __shared__ float2 cs[kMaxHalf];
  __shared__ int s_pages[kSmemPages];
  __shared__ __align__(8) uint64_t bars[kCopyWarps][kRing];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t unit_bytes = uint32_t(kPage) * D * 2;  // one slot
  uint8_t* ring = ring_raw + size_t(warp) * kRing * unit_bytes;
  if (lane == 0)
    for (int r = 0; r < kRing; ++r) mbar_init(&bars[warp][r], 1);
  fence_barrier_init();
  pdl_wait();  // the chunk tables and pages come from the work before (dependent launch)
  pdl_launch_next();
  const int32_t* meta = chunk_meta + blockIdx.y * CKV_META_STRIDE;
  const int table_off = meta[CKV_META_TABLE_OFFSET];
  const int length = meta[CKV_META_LENGTH];
  const int dst_start = meta[CKV_META_DST_START];
  const int delta = meta[CKV_META_DELTA];
  const int lb = max(layer_lo, meta[CKV_META_LAYER_BEGIN]);
  const int le = min(layer_hi, meta[CKV_META_LAYER_END]);
  const int src_off = meta[CKV_META_SRC_OFFSET];
  if (le <= lb || length <= 0) return;  // the whole CTA: nothing issued yet
  const bool rotate = delta != 0;
  if (rotate)
    for (int j = threadIdx.x; j < rot / 2; j += blockDim.x) cs[j] = rope_cs(float(delta), inv_freq[j]);
  const int n_slots = min(kSmemPages, (src_off + length + kPage - 1) / kPage);
  for (int i = threadIdx.x; i < n_slots; i += blockDim.x) s_pages[i] = page_table[table_off + i];
  __syncthreads();

  const int nl = le - lb;
  const int n_blocks = (length + kPage - 1) / kPage;
  const int n_units = n_blocks * nl * 2 * H;  // < 2^31: checked on the host
  const int64_t layer_elems = int64_t(H) * n_ctx * D;
  const int first = blockIdx.x * kCopyWarps + warp, step = gridDim.x * kCopyWarps;
  const int my_units = first < n_units ? (n_units - 1 - first) / step + 1 : 0;

  // where unit k of this warp comes from (up to two page pieces) and goes to
  struct Unit {
    const uint16_t* src[2];
    int rows[2];  // rows of each piece (0: none, or skipped for a bad page id)
    int off[2];   // row offset of each piece in the unit (and in the slot)
    int n;        // rows of the unit
    uint16_t* dst;
    bool rot;
  };
  auto unit = [&](int k) {
    Unit x{{nullptr, nullptr}, {0, 0}, {0, 0}, 0, nullptr, false};
    int t = first + k * step;
    const int b = t % n_blocks;
    t /= n_blocks;
    const int h = t % H;
    t /= H;
    const int kv = t & 1;
    t >>= 1;
    const int l = lb + t;
    const int r0 = b * kPage;
    const int rows = min(kPage, length - r0);
    const int dpos = dst_start + r0;
    if (dpos < 0 || dpos + rows > n_ctx) {
      if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
      return x;
    }
    x.dst = (kv ? v_out : k_out) + int64_t(l - layer_lo) * layer_elems + (int64_t(h) * n_ctx + dpos) * D;
    x.rot = rotate && kv == 0;
    int done = 0;
    for (int piece = 0; piece < 2 && done < rows; ++piece) {
      const int tok = src_off + r0 + done;
      const int slot = tok / kPage, in_page = tok % kPage;
      const int take = min(rows - done, kPage - in_page);
      const int page = slot < kSmemPages ? s_pages[slot] : page_table[table_off + slot];
      x.off[piece] = done;
      if (page < 0 || page >= n_pages) {
        if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_PAGE_RANGE);
      } else {
        x.src[piece] = pool + ((((int64_t(page) * n_layers + l) * 2 + kv) * H + h) * kPage + in_page) * D;
        x.rows[piece] = take;
      }
      done += take;
    }
    x.n = rows;
    return x;
  };
  // lane 0: the copies of unit k into slot k % kRing (pieces at their row offsets)
  auto load = [&](int k, const Unit& x) {
    uint64_t* bar = &bars[warp][k % kRing];
    uint8_t* slot = ring + (k % kRing) * unit_bytes;
    const uint32_t b0 = uint32_t(x.rows[0]) * D * 2, b1 = uint32_t(x.rows[1]) * D * 2;
    if (b0 + b1 == 0) {
      mbar_arrive(bar);  // nothing to copy: the slot's phase completes at once
      return;
    }
    mbar_expect_tx(bar, b0 + b1);
    if (b0) bulk_load(slot + uint32_t(x.off[0]) * D * 2, x.src[0], b0, bar);
    if (b1) bulk_load(slot + uint32_t(x.off[1]) * D * 2, x.src[1], b1, bar);
  };
  if (lane == 0)
    for (int k = 0; k < kRing - 1 && k < my_units; ++k) load(k, unit(k));
  for (int k = 0; k < my_units; ++k) {
    const Unit x = unit(k);
    uint8_t* slot = ring + (k % kRing) * unit_bytes;
    // this unit's copies have landed (every lane waits: the lanes read the slot)
    const uint64_t t0 = global_ns();
    bool ok = true;
    while (!mbar_try_wait(&bars[warp][k % kRing], (k / kRing) & 1))
      if (global_ns() - t0 > kWaitLimitNs) {
        ok = false;
        break;
      }
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) {
        atomicOr(&g_err_word, CKV_DEV_ERR_WAIT_TIMEOUT);
        // let the copies already issued (units k .. k + kRing - 2) land before the CTA goes
        for (int j = k; j < k + kRing - 1 && j < my_units; ++j) {
          const uint64_t t1 = global_ns();
          while (!mbar_try_wait(&bars[warp][j % kRing], (j / kRing) & 1))
            if (global_ns() - t1 > kWaitLimitNs) break;
        }
      }
      break;
    }
    const int rows = x.n;
    if (x.rot && rows > 0) {
      // rotate in place: lane takes rotary pairs (vectors p and p + rot / 16 of a row) and
      // writes them back to the same slot positions
      uint4* st = reinterpret_cast<uint4*>(slot);
      const int vec_row = D / 8, n_pair = rot / 16;
      for (int it = lane; it < kPage * n_pair; it += 32) {
        const int r = it / n_pair, item = it - r * n_pair;
        if (r >= rows) break;
        const int base = r * vec_row;
        uint4 v1 = st[base + item], v2 = st[base + item + n_pair];
        rotate8(v1, v2, cs + item * 8);
        st[base + item] = v1;
        st[base + item + n_pair] = v2;
      }
      fence_async_smem();
    }
    __syncwarp();
    if (lane == 0) {
      // the slot's rows out to the blended cache (per piece: a skipped piece keeps dst
      // untouched), then the copies of unit k + kRing - 1 into the slot unit k - 1 used
#pragma unroll
      for (int piece = 0; piece < 2; ++piece)
        if (x.rows[piece])
          bulk_store(x.dst + int64_t(x.off[piece]) * D, slot + uint32_t(x.off[piece]) * D * 2,
                     uint32_t(x.rows[piece]) * D * 2);
      bulk_commit();
      if (k + kRing - 1 < my_units) {
        bulk_wait_read<1>();  // the store of unit k - 1 has read its slot
        load(k + kRing - 1, unit(k + kRing - 1));
      }
    }
    __syncwarp();
  }
  if (lane == 0) bulk_wait_all();  // the stores have written the cache before the CTA ends
}

// Dense (H, >=length, D) per-layer sources -> pages.
__global__ void __launch_bounds__(256) pages_write_kernel(
    uint16_t* __restrict__ pool, int64_t n_pages, const int32_t* __restrict__ page_ids, int length,
    const uint64_t* __restrict__ k_ptrs, const uint64_t* __restrict__ v_ptrs, int64_t head_stride,
    int n_layers, int H, int D) {
  __shared__ __align__(16) uint4 s_stage[kCopyWarps][kStageVec];
  pdl_wait();  // the chunk's K/V come from the kernels before (dependent launch)
  pdl_launch_next();
  const int n_blocks = (length + kPage - 1) / kPage;
  const int64_t n_units = int64_t(n_blocks) * n_layers * 2 * H;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int warps = blockDim.x / 32;
  for (int64_t u = int64_t(blockIdx.x) * warps + warp; u < n_units; u += int64_t(gridDim.x) * warps) {
    int64_t t = u;
    const int h = int(t % H);
    t /= H;
    const int kv = int(t % 2);
    t /= 2;
    const int l = int(t % n_layers);
    const int b = int(t / n_layers);
    const int page = page_ids[b];
    if (page < 0 || page >= n_pages) {
      if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_PAGE_RANGE);
      continue;
    }
    const int r0 = b * kPage;
    const int rows = min(kPage, length - r0);
    const uint64_t base = (kv ? v_ptrs : k_ptrs)[l];
    if ((base & 15u) != 0) {
      if (lane == 0) atomicOr(&g_err_word, CKV_DEV_ERR_POSITION_RANGE);
      continue;
    }
    const uint16_t* src = reinterpret_cast<const uint16_t*>(base) + h * head_stride + int64_t(r0) * D;
    uint16_t* dst = pool + (((int64_t(page) * n_layers + l) * 2 + kv) * H + h) * kPage * D;
    copy_flat_warp(reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), rows * (D / 8),
                   s_stage[warp], lane);
  }
}

int check_rot(int head_dim, int rot) {
  CKV_REQUIRE(head_dim > 0 && head_dim % 8 == 0 && head_dim <= 2 * kMaxHalf,
              "head_dim %d must be a positive multiple of 8 and <= %d", head_dim, 2 * kMaxHalf);
  CKV_REQUIRE(rot > 0 && rot % 16 == 0 && rot <= head_dim,
              "rot_dims %d must be a positive multiple of 16 and <= head_dim", rot);
  return CKV_OK;
}

}  // namespace
}  // namespace ckv

using namespace ckv;

extern "C" {

int ckv_rope_table(const float* inv_freq, int half_dim, int max_pos, float* table,
                   ckv_stream_t stream) {
  CKV_REQUIRE(inv_freq && table, "ckv_rope_table: null pointer");
  CKV_REQUIRE(half_dim > 0 && max_pos > 0, "ckv_rope_table: bad sizes");
  const int64_t n = int64_t(half_dim) * max_pos;
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * num_sms()));
  rope_table_kernel<<<grid, 256, 0, as_stream(stream)>>>(inv_freq, half_dim, max_pos,
                                                         reinterpret_cast<float2*>(table));
  CKV_LAUNCH_CHECK("ckv_rope_table");
  return CKV_OK;
}

int ckv_shift_keys(const uint16_t* src, uint16_t* dst, int64_t rows, int head_dim, int rot_dims,
                   int delta, const float* inv_freq, ckv_stream_t stream) {
  CKV_REQUIRE(src && dst && inv_freq, "ckv_shift_keys: null pointer");
  CKV_REQUIRE(aligned16(src) && aligned16(dst), "ckv_shift_keys: pointers must be 16-byte aligned");
  if (int rc = check_rot(head_dim, rot_dims)) return rc;
  if (rows <= 0) return CKV_OK;
  if (delta == 0) {
    if (src != dst)
      if (cudaMemcpyAsync(dst, src, rows * head_dim * 2, cudaMemcpyDeviceToDevice,
                          as_stream(stream)) != cudaSuccess) {
        set_error("ckv_shift_keys: copy failed");
        return CKV_ERR_CUDA;
      }
    return CKV_OK;
  }
  const int64_t units = (rows + kPage - 1) / kPage;
  const int grid = int(std::min<int64_t>((units + 7) / 8, 4 * num_sms()));
  launch_pdl(shift_rows_kernel, dim3(grid), dim3(256), 0, as_stream(stream), src, dst, rows, head_dim, rot_dims,
             delta, inv_freq);
  CKV_LAUNCH_CHECK("ckv_shift_keys");
  return CKV_OK;
}

int ckv_apply_rope(const uint16_t* src, uint16_t* dst, int64_t batch_heads, int seq, int head_dim,
                   int rot_dims, const int32_t* positions, const float* inv_freq,
                   ckv_stream_t stream) {
  CKV_REQUIRE(src && dst && inv_freq && positions, "ckv_apply_rope: null pointer");
  CKV_REQUIRE(aligned16(src) && aligned16(dst), "ckv_apply_rope: pointers must be 16-byte aligned");
  if (int rc = check_rot(head_dim, rot_dims)) return rc;
  CKV_REQUIRE(seq >= 0 && batch_heads >= 0, "ckv_apply_rope: bad sizes");
  const int64_t rows = batch_heads * seq;
  if (rows == 0) return CKV_OK;
  const int64_t items = rows * (head_dim / 8 - rot_dims / 16);
  const int grid = static_cast<int>(std::min<int64_t>((items + 255) / 256, 16 * num_sms()));
  rope_rows_kernel<<<grid, 256, 0, as_stream(stream)>>>(src, dst, rows, head_dim, rot_dims, 0,
                                                        positions, seq, inv_freq);
  CKV_LAUNCH_CHECK("ckv_apply_rope");
  return CKV_OK;
}

int ckv_shift_keys_f32(const float* src, float* dst, int64_t rows, int head_dim, int rot_dims, int delta,
                       const float* inv_freq, ckv_stream_t stream) {
  CKV_REQUIRE(src && dst && inv_freq, "ckv_shift_keys_f32: null pointer");
  CKV_REQUIRE(aligned16(src) && aligned16(dst), "ckv_shift_keys_f32: pointers must be 16-byte aligned");
  if (int rc = check_rot(head_dim, rot_dims)) return rc;
  if (rows <= 0) return CKV_OK;
  if (delta == 0) {
    if (src != dst && cudaMemcpyAsync(dst, src, rows * head_dim * 4, cudaMemcpyDeviceToDevice,
                                      as_stream(stream)) != cudaSuccess) {
      set_error("ckv_shift_keys_f32: copy failed");
      return CKV_ERR_CUDA;
    }
    return CKV_OK;
  }
  return launch_rope_f32(src, dst, rows, head_dim, rot_dims, delta, nullptr, 1, inv_freq, as_stream(stream),
                         "ckv_shift_keys_f32");
}

int ckv_apply_rope_f32(const float* src, float* dst, int64_t batch_heads, int seq, int head_dim, int rot_dims,
                       const int32_t* positions, const float* inv_freq, ckv_stream_t stream) {
  CKV_REQUIRE(src && dst && inv_freq && positions, "ckv_apply_rope_f32: null pointer");
  CKV_REQUIRE(aligned16(src) && aligned16(dst), "ckv_apply_rope_f32: pointers must be 16-byte aligned");
  if (int rc = check_rot(head_dim, rot_dims)) return rc;
  CKV_REQUIRE(seq >= 0 && batch_heads >= 0, "ckv_apply_rope_f32: bad sizes");
  const int64_t rows = batch_heads * seq;
  if (rows == 0) return CKV_OK;
  return launch_rope_f32(src, dst, rows, head_dim, rot_dims, 0, positions, seq, inv_freq, as_stream(stream),
                         "ckv_apply_rope_f32");
}

static int gather_common(const int32_t* chunk_meta, int n_chunks, const float* inv_freq, int rot,
                         uint16_t* k_out, uint16_t* v_out, int layer_lo, int layer_hi, int H, int D,
                         int n_ctx) {
  CKV_REQUIRE(chunk_meta && inv_freq && k_out && v_out, "blend_gather: null pointer");
  CKV_REQUIRE(aligned16(k_out) && aligned16(v_out), "blend_gather: outputs must be 16-byte aligned");
  if (int rc = check_rot(D, rot)) return rc;
  CKV_REQUIRE(n_chunks >= 0 && n_chunks <= 65535, "blend_gather: n_chunks %d out of range", n_chunks);
  CKV_REQUIRE(layer_lo >= 0 && layer_hi >= layer_lo, "blend_gather: bad layer range");
  CKV_REQUIRE(H > 0 && n_ctx > 0, "blend_gather: bad sizes");
  CKV_REQUIRE(int64_t((n_ctx + kPage - 1) / kPage) * (layer_hi - layer_lo) * 2 * H < (int64_t(1) << 31),
              "blend_gather: too many (page, layer, K|V, head) units for one launch");
  return CKV_OK;
}

int ckv_blend_gather_paged(const uint16_t* pool, int64_t n_pages, const int32_t* page_table,
                           const int32_t* chunk_meta, int n_chunks, const float* inv_freq,
                           int rot_dims, uint16_t* k_out, uint16_t* v_out, int layer_lo,
                           int layer_hi, int n_layers, int n_kv_heads, int head_dim, int n_ctx,
                           ckv_stream_t stream) {
  if (int rc = gather_common(chunk_meta, n_chunks, inv_freq, rot_dims, k_out, v_out, layer_lo,
                             layer_hi, n_kv_heads, head_dim, n_ctx))
    return rc;
  CKV_REQUIRE(pool && page_table && aligned16(pool), "ckv_blend_gather_paged: bad pool/page table");
  CKV_REQUIRE(layer_hi <= n_layers, "ckv_blend_gather_paged: layer_hi > n_layers");
  if (n_chunks == 0 || layer_hi == layer_lo) return CKV_OK;
  // the TMA ring: kRing slots of one 16-token unit per warp (96 KiB per CTA at head_dim
  // 128, two CTAs per SM)
  const int smem = kCopyWarps * kRing * kPage * head_dim * 2;
  if (int rc = set_smem_limit(reinterpret_cast<const void*>(blend_gather_bulk_kernel), smem)) return rc;
  const int gx = std::max(1, 2 * num_sms() / n_chunks);
  launch_pdl(blend_gather_bulk_kernel, dim3(gx, n_chunks), dim3(256), smem, as_stream(stream), pool, n_pages,
             page_table, chunk_meta, inv_freq, rot_dims, k_out, v_out, layer_lo, layer_hi, n_layers, n_kv_heads,
             head_dim, n_ctx);
  CKV_LAUNCH_CHECK("ckv_blend_gather_paged");
  return CKV_OK;
}

int ckv_blend_gather_dense(const uint64_t* k_ptrs, const uint64_t* v_ptrs,
                           const int32_t* chunk_meta, int n_chunks, const float* inv_freq,
                           int rot_dims, uint16_t* k_out, uint16_t* v_out, int layer_lo,
                           int layer_hi, int n_kv_heads, int head_dim, int n_ctx,
                           ckv_stream_t stream) {
  if (int rc = gather_common(chunk_meta, n_chunks, inv_freq, rot_dims, k_out, v_out, layer_lo,
                             layer_hi, n_kv_heads, head_dim, n_ctx))
    return rc;
  CKV_REQUIRE(k_ptrs && v_ptrs, "ckv_blend_gather_dense: null pointer arrays");
  if (n_chunks == 0 || layer_hi == layer_lo) return CKV_OK;
  const int gx = std::max(1, 4 * num_sms() / n_chunks);
  launch_pdl(blend_gather_kernel<false>, dim3(gx, n_chunks), dim3(256), 0, as_stream(stream),
             static_cast<const uint16_t*>(nullptr), int64_t(0), static_cast<const int32_t*>(nullptr), k_ptrs,
             v_ptrs, chunk_meta, inv_freq, rot_dims, k_out, v_out, layer_lo, layer_hi, /*n_layers=*/0,
             n_kv_heads, head_dim, n_ctx);
  CKV_LAUNCH_CHECK("ckv_blend_gather_dense");
  return CKV_OK;
}

int ckv_pages_write(uint16_t* pool, int64_t n_pages, const int32_t* page_ids, int length,
                    const uint64_t* k_ptrs, const uint64_t* v_ptrs, int64_t head_stride,
                    int n_layers, int n_kv_heads, int head_dim, ckv_stream_t stream) {
  CKV_REQUIRE(pool && page_ids && k_ptrs && v_ptrs, "ckv_pages_write: null pointer");
  CKV_REQUIRE(aligned16(pool), "ckv_pages_write: pool must be 16-byte aligned");
  CKV_REQUIRE(head_dim > 0 && head_dim % 8 == 0, "ckv_pages_write: head_dim %% 8 != 0");
  CKV_REQUIRE(n_layers > 0 && n_kv_heads > 0 && length >= 0, "ckv_pages_write: bad sizes");
  CKV_REQUIRE(head_stride % 8 == 0, "ckv_pages_write: head_stride must keep 16-byte alignment");
  if (length == 0) return CKV_OK;
  const int64_t units = int64_t(ceil_div(length, kPage)) * n_layers * 2 * n_kv_heads;
  const int grid = static_cast<int>(std::min<int64_t>((units + 7) / 8, 8 * num_sms()));
  launch_pdl(pages_write_kernel, dim3(grid), dim3(256), 0, as_stream(stream), pool, n_pages, page_ids, length,
             k_ptrs, v_ptrs, head_stride, n_layers, n_kv_heads, head_dim);
  CKV_LAUNCH_CHECK("ckv_pages_write");
  return CKV_OK;
}

}  // extern "C"
