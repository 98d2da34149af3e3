// Causal paged prefill attention for prompt chunks (the varlen branch of the reference's
// paged attention, transformers integrations/flash_paged.py:50-81, after cache.update).
//
// A tile is up to 64 consecutive prompt rows of one request and one head. Its queries attend
// to keys [0, pos_start + nrows) of that request through the block table (the chunk's own K/V
// was written by cdb_rope_append_kv first), causally. Each CTA (4 warps x 16 query rows) keeps
// Q in registers, streams 64-key K/V tiles (4 pages) through a double-buffered, XOR-swizzled
// shared-memory ring with cp.async, and runs QK^T and PV on the tensor cores (bf16 mma.sync,
// fp32 accumulation) with a base-2 online softmax in registers. Every K/V page is read once per
// 64 queries instead of once per query.
#include "cdb_common.cuh"

namespace cdb {
namespace prefill {

constexpr int TQ = 64;  // query rows per tile
constexpr int TK = 64;  // keys per tile (4 pages of 16)
constexpr int kBlock = 16;
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  const __nv_bfloat16* qkv;
  int64_t qkv_stride, k_col, v_col;
  __nv_bfloat16* out;
  int64_t out_stride;
  const __nv_bfloat16* kv;
  int64_t kv_rows;
  int cache_layer;
  const int32_t* block_table;
  int64_t bt_stride;
  const int4* tiles;  // {row_start, nrows, slot, pos_start}
  int num_heads;
  float scale_log2;
  int32_t* status;
};

// Shared-memory row pitch of a [rows][D] bf16 tile. D = 64/128: rows of D*2 bytes with the
// 16-byte chunk index XOR-swizzled by r % 8 (rows hold whole groups of 8 chunks). D = 96: 12
// chunks per row do not form whole groups, so rows are padded to 13 chunks (208 bytes) instead;
// the 8 rows one ldmatrix phase reads then start in distinct bank groups ((13 r + c) mod 8).
template <int D>
struct RowPitch {
  static constexpr int BYTES = (D == 96) ? 208 : D * 2;
  static constexpr bool XOR = (D != 96);
};

template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * RowPitch<D>::BYTES + ((RowPitch<D>::XOR ? (c ^ (r & 7)) : c) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int D>
__global__ void __launch_bounds__(128, 3) prefill_attn_kernel(Params p) {
  pdl_trigger();
  pdl_wait();
  constexpr int NCH = D / 8;   // 16-byte chunks per row
  constexpr int KS = D / 16;   // k-steps over the head dim
  constexpr int NT = D / 8;    // n-tiles of the output
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int PITCH = RowPitch<D>::BYTES;
  uint8_t* sk = smem;                       // [2][TK][D]
  uint8_t* sv = sk + 2 * TK * PITCH;        // [2][TK][D]
  // Q is staged in the second K buffer (TQ == TK rows), which the first prefetch overwrites only
  // after every warp holds its Q fragments in registers: 64 KB of shared memory instead of 80, so
  // three CTAs share an SM.
  static_assert(TQ == TK, "Q borrows a K buffer");
  uint8_t* sq = sk + TK * PITCH;
  const uint32_t sq_u = smem_u32(sq), sk_u = smem_u32(sk), sv_u = smem_u32(sv);

  const int4 tile = p.tiles[blockIdx.y];  // heads vary fastest: a tile's heads launch together
  const int head = blockIdx.x;
  const int row0 = tile.x, nrows = tile.y, slot = tile.z, pos0 = tile.w;
  const int kv_len = pos0 + nrows;
  const int n_kt = (kv_len + TK - 1) / TK;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int32_t* bt = p.block_table + (int64_t)slot * p.bt_stride;
  const int64_t hstride = (int64_t)p.num_heads * D;
  const __nv_bfloat16* kbase = p.kv + (int64_t)(2 * p.cache_layer) * p.kv_rows * hstride + (int64_t)head * D;
  const __nv_bfloat16* vbase = p.kv + (int64_t)(2 * p.cache_layer + 1) * p.kv_rows * hstride + (int64_t)head * D;

  // Q tile -> shared (zero rows past nrows)
  for (int i = tid; i < TQ * NCH; i += 128) {
    const int r = i / NCH, c = i % NCH;
    const __nv_bfloat16* src = p.qkv + (int64_t)(row0 + min(r, nrows - 1)) * p.qkv_stride + (int64_t)head * D + c * 8;
    cp_async16(sq_u + swz<D>(r, c), src, r < nrows);
  }
  auto load_kv = [&](int kt, int buf) {
    for (int i = tid; i < TK * NCH; i += 128) {
      const int r = i / NCH, c = i % NCH;
      const int key = kt * TK + r;
      const bool valid = key < kv_len;
      int64_t row = 0;
      if (valid) {
        const int blk = bt[key / kBlock];
        row = (int64_t)blk * kBlock + key % kBlock;
        if (blk < 0 || row >= p.kv_rows) row = 0;
      }
      const uint32_t off = (uint32_t)(buf * TK * PITCH) + swz<D>(r, c);
      cp_async16(sk_u + off, kbase + row * hstride + c * 8, valid);
      cp_async16(sv_u + off, vbase + row * hstride + c * 8, valid);
    }
  };
  load_kv(0, 0);
  cp_commit();

  // Q fragments for this warp's 16 rows.
  cp_wait<0>();
  __syncthreads();
  uint32_t qa[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
    const int c = 2 * kk + (lane >> 4);
    ldsm_x4(sq_u + swz<D>(r, c), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
  }
  __syncthreads();  // every warp has its Q fragments: the K buffer holding Q may be refilled

  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  const int qr_a = warp * 16 + (lane >> 2);
  const int qpos_a = pos0 + qr_a, qpos_b = qpos_a + 8;

  for (int kt = 0; kt < n_kt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kt) load_kv(kt + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const uint32_t kb = sk_u + (uint32_t)(buf * TK * PITCH);
    const uint32_t vb = sv_u + (uint32_t)(buf * TK * PITCH);

    float s[TK / 8][4];
#pragma unroll
    for (int j = 0; j < TK / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
      for (int np = 0; np < TK / 16; ++np) {
        const int r = np * 16 + (lane & 7) + 8 * (lane >> 4);
        const int c = 2 * kk + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + swz<D>(r, c), b0, b1, b2, b3);
        mma16816(s[2 * np], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
        mma16816(s[2 * np + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
      }
    }
    // scale, causal / length mask, online softmax (rows a = lane/4, b = a + 8)
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int j = 0; j < TK / 8; ++j) {
      const int key = kt * TK + j * 8 + 2 * (lane & 3);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kp = key + e;
        const bool ok_a = kp <= qpos_a && kp < kv_len;
        const bool ok_b = kp <= qpos_b && kp < kv_len;
        s[j][e] = ok_a ? s[j][e] * p.scale_log2 : -INFINITY;
        s[j][2 + e] = ok_b ? s[j][2 + e] * p.scale_log2 : -INFINITY;
        mx_a = fmaxf(mx_a, s[j][e]);
        mx_b = fmaxf(mx_b, s[j][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
    }
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float al_a = (mn_a == -INFINITY) ? 1.f : exp2f(m_a - mn_a);
    const float al_b = (mn_b == -INFINITY) ? 1.f : exp2f(m_b - mn_b);
    m_a = mn_a;
    m_b = mn_b;
    float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
    for (int j = 0; j < TK / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[j][e] = (s[j][e] == -INFINITY) ? 0.f : exp2f(s[j][e] - mn_a);
        s[j][2 + e] = (s[j][2 + e] == -INFINITY) ? 0.f : exp2f(s[j][2 + e] - mn_b);
        sum_a += s[j][e];
        sum_b += s[j][2 + e];
      }
    }
    l_a = l_a * al_a + sum_a;
    l_b = l_b * al_b + sum_b;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      o[j][0] *= al_a;
      o[j][1] *= al_a;
      o[j][2] *= al_b;
      o[j][3] *= al_b;
    }
    // O += P V
#pragma unroll
    for (int kk2 = 0; kk2 < TK / 16; ++kk2) {
      const uint32_t a0 = pack_bf16x2(s[2 * kk2][0], s[2 * kk2][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * kk2][2], s[2 * kk2][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * kk2 + 1][0], s[2 * kk2 + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * kk2 + 1][2], s[2 * kk2 + 1][3]);
#pragma unroll
      for (int cp = 0; cp < NT / 2; ++cp) {
        const int r = kk2 * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int c = 2 * cp + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + swz<D>(r, c), b0, b1, b2, b3);
        mma16816(o[2 * cp], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * cp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();

#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
  }
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f;
  const float inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  const int ra = qr_a, rb = qr_a + 8;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int col = head * D + j * 8 + 2 * (lane & 3);
    if (ra < nrows)
      *reinterpret_cast<uint32_t*>(p.out + (int64_t)(row0 + ra) * p.out_stride + col) =
          pack_bf16x2(o[j][0] * inv_a, o[j][1] * inv_a);
    if (rb < nrows)
      *reinterpret_cast<uint32_t*>(p.out + (int64_t)(row0 + rb) * p.out_stride + col) =
          pack_bf16x2(o[j][2] * inv_b, o[j][3] * inv_b);
  }
}

template <int D>
static int launch(const Params& p, int num_tiles, cudaStream_t st) {
  constexpr int SMEM = 4 * TK * RowPitch<D>::BYTES;  // K and V double buffers (Q borrows one)
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(prefill_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) !=
        cudaSuccess)
      return CDB_ERR_CUDA;
    attr = true;
  }
  if (num_tiles > 65535) return CDB_ERR_INVALID_ARGUMENT;  // grid y
  dim3 grid(p.num_heads, num_tiles);
  launch_pdl(prefill_attn_kernel<D>, dim3(grid), dim3(128), SMEM, st, p);
  return cudaPeekAtLastError() == cudaSuccess ? CDB_OK : CDB_ERR_CUDA;
}

}  // namespace prefill
}  // namespace cdb

extern "C" int cdb_prefill_attention(const void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col, void* out,
                                     int64_t out_stride, const void* kv_base, int num_cache_layers, int64_t kv_rows,
                                     int cache_layer, const int32_t* block_table, int64_t block_table_stride,
                                     const void* tiles, int num_tiles, int num_heads, int head_dim, int block_size,
                                     float scale, int32_t* status, void* stream) {
  using namespace cdb::prefill;
  if (block_size != kBlock || cache_layer < 0 || cache_layer >= num_cache_layers || num_tiles < 0 || num_heads <= 0)
    return CDB_ERR_INVALID_ARGUMENT;
  if ((qkv_stride & 7) || (k_col & 7) || (v_col & 7) || (out_stride & 1)) return CDB_ERR_INVALID_ARGUMENT;
  if (num_tiles == 0) return CDB_OK;
  Params p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.qkv_stride = qkv_stride;
  p.k_col = k_col;
  p.v_col = v_col;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.kv = static_cast<const __nv_bfloat16*>(kv_base);
  p.kv_rows = kv_rows;
  p.cache_layer = cache_layer;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.tiles = static_cast<const int4*>(tiles);
  p.num_heads = num_heads;
  p.scale_log2 = scale * kLog2e;
  p.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 128) return launch<128>(p, num_tiles, st);
  if (head_dim == 64) return launch<64>(p, num_tiles, st);
  if (head_dim == 96) return launch<96>(p, num_tiles, st);
  return CDB_ERR_UNSUPPORTED;
}
