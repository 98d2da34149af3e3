// Ragged-depth paged decode attention for sm_100a.
//
// One launch serves one cache layer of a recurrent (or prefill) launch whose rows sit at
// different positions and recurrent steps. Work is split into units (row, head group,
// KV split) by cdb_attn_plan so CTAs see roughly equal byte counts despite ragged contexts.
//
// Each CTA is warp specialised: one producer warp streams K and V pages of the unit
// through a NSTAGE-deep shared-memory ring with 4-D TMA tile loads (one 16-token x HG-head x
// D tile per page, completion on an mbarrier); HG consumer warps, one per head, do the
// QK dot products, the online softmax and the PV accumulation in fp32 from shared memory.
// The appended token's k/v never round-trip through the cache: the unit holding the last
// split rotates k, folds the new token in from registers and writes k/v to its cache row.
// Splits of one (row, head group) combine through scratch: the last CTA to finish (atomic
// counter) merges the partial (m, l, o) triples and resets its counter.
#include <cuda.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "cdb_common.cuh"

namespace cdb {

constexpr int kMaxSplits = 64;
constexpr int kBlock = 16;  // tokens per page (block_size)
constexpr float kLog2e = 1.4426950408889634f;

template <int D, int HG>
struct AttnCfg {
  static constexpr int NSTAGE = 3;
  static constexpr int LPT = (D == 96) ? 4 : 8;  // lanes cooperating on one token's QK dot
  static constexpr int DPL = D / LPT;            // dims per lane in QK
  static constexpr int TPP = 32 / LPT;           // tokens per pass
  static constexpr int PASSES = kBlock / TPP;
  static constexpr int NPAIR = D / 2;
  static constexpr int PPL = (NPAIR + 31) / 32;  // bf16 pairs per lane in PV
  static constexpr int NCH = DPL / 8;          // 16-byte chunks per lane; lane cq owns chunks cq + c*LPT
  static constexpr int TILE_BYTES = kBlock * HG * D * 2;
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int THREADS = (HG + 1) * 32;
  static constexpr int SMEM = NSTAGE * STAGE_BYTES + 2 * NSTAGE * 8 + 64;
  static_assert(DPL % 8 == 0, "QK lane slice must be whole 16-byte chunks");
};

struct AttnParams {
  const __nv_bfloat16* qkv;
  int64_t qkv_stride, k_col, v_col;
  __nv_bfloat16* out;
  int64_t out_stride;
  __nv_bfloat16* kv;
  int64_t kv_rows;
  int cache_layer;
  const int32_t* block_table;
  int64_t bt_stride;
  const int32_t* item_slot;
  const int32_t* item_pos;
  int rope_mode;
  const void* rope_cos;
  const void* rope_sin;
  int append;
  const int32_t* hdr;
  const int4* units;
  float* part_o;
  float* part_ml;
  int32_t* counters;
  int num_heads;
  float scale_log2;
  int32_t* status;
};

// Rotated value of element d of one head vector (Ouro split-half rotate_half RoPE with
// bf16 cos/sin, every product and the sum rounded to bf16 as PyTorch's bf16 ops round).
__device__ __forceinline__ float rope_elem(const __nv_bfloat16* x, int d, int D, const __nv_bfloat16* cos_row,
                                           const __nv_bfloat16* sin_row) {
  const int half = D / 2;
  const float xv = bf16_to_f(x[d]);
  const float rot = d < half ? -bf16_to_f(x[d + half]) : bf16_to_f(x[d - half]);
  const float a = round_bf16(xv * bf16_to_f(cos_row[d]));
  const float b = round_bf16(rot * bf16_to_f(sin_row[d]));
  return round_bf16(a + b);
}

// Huginn interleaved-pair rotation in fp32 (modeling_huginn.py:178-196): pairs (2i, 2i+1).
__device__ __forceinline__ float rope_elem_pairs(const __nv_bfloat16* x, int d, const float* cos_row,
                                                 const float* sin_row) {
  const int i = d >> 1;
  const float x0 = bf16_to_f(x[2 * i]);
  const float x1 = bf16_to_f(x[2 * i + 1]);
  const float c = cos_row[i], s = sin_row[i];
  return round_bf16((d & 1) ? (x0 * s + x1 * c) : (x0 * c - x1 * s));
}

template <int D>
__device__ __forceinline__ float load_rot(const AttnParams& p, const __nv_bfloat16* x, int d, int pos) {
  if (p.rope_mode == 1) {
    const __nv_bfloat16* c = static_cast<const __nv_bfloat16*>(p.rope_cos) + (int64_t)pos * D;
    const __nv_bfloat16* s = static_cast<const __nv_bfloat16*>(p.rope_sin) + (int64_t)pos * D;
    return rope_elem(x, d, D, c, s);
  }
  if (p.rope_mode == 2) {
    const float* c = static_cast<const float*>(p.rope_cos) + (int64_t)pos * (D / 2);
    const float* s = static_cast<const float*>(p.rope_sin) + (int64_t)pos * (D / 2);
    return rope_elem_pairs(x, d, c, s);
  }
  return bf16_to_f(x[d]);
}

template <int D, int HG>
__global__ void __launch_bounds__(AttnCfg<D, HG>::THREADS) decode_attn_kernel(const __grid_constant__ CUtensorMap map,
                                                                              AttnParams p) {
  using C = AttnCfg<D, HG>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NSTAGE * C::STAGE_BYTES);
  uint64_t* empty = full + C::NSTAGE;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], HG);
    }
    fence_barrier_init();
  }
  __syncthreads();

  const int n_units = p.hdr[0];
  const int sb = p.hdr[1];
  if (warp == HG) {
    // ------------------------------------------------------------- producer warp
    if (lane == 0) {
      prefetch_tensormap(&map);
      int stage = 0;
      uint32_t phase = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const int4 unit = p.units[u];
        const int pos = p.item_pos[unit.x];
        const int n_cached = p.append ? pos : pos + 1;
        const int nb = (n_cached + kBlock - 1) / kBlock;
        const int b0 = unit.z * sb;
        const int b1 = min(b0 + sb, nb);
        const int32_t* bt = p.block_table + (int64_t)p.item_slot[unit.x] * p.bt_stride;
        for (int blk = b0; blk < b1; ++blk) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) return;
          const int block_id = bt[blk];
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          uint8_t* dst = smem + stage * C::STAGE_BYTES;
          tma_load_4d(dst, &map, &full[stage], 0, unit.y * HG, block_id * kBlock, 2 * p.cache_layer);
          tma_load_4d(dst + C::TILE_BYTES, &map, &full[stage], 0, unit.y * HG, block_id * kBlock,
                      2 * p.cache_layer + 1);
          if (++stage == C::NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    return;
  }

  // --------------------------------------------------------------- consumer warps
  const int hh = warp;            // head within the group
  const int tq = lane / C::LPT;   // token slot within a pass
  const int cq = lane % C::LPT;   // dim slice within the token
  int stage = 0;
  uint32_t phase = 0;

  for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
    const int4 unit = p.units[u];
    const int item = unit.x;
    const int head = unit.y * HG + hh;
    const int split = unit.z;
    const int nsplit = unit.w;
    const int pos = p.item_pos[item];
    const int n_cached = p.append ? pos : pos + 1;
    const int nb = (n_cached + kBlock - 1) / kBlock;
    const int b0 = split * sb;
    const int b1 = min(b0 + sb, nb);

    // q slice for this lane (rotated when RoPE is fused), pre-scaled by softmax_scale*log2(e).
    const __nv_bfloat16* qrow = p.qkv + (int64_t)item * p.qkv_stride + (int64_t)head * D;
    float qf[C::DPL];
#pragma unroll
    for (int i = 0; i < C::DPL; ++i) {
      const int d = ((i / 8) * C::LPT + cq) * 8 + (i % 8);
      qf[i] = (p.append ? load_rot<D>(p, qrow, d, pos) : bf16_to_f(qrow[d])) * p.scale_log2;
    }

    float m = -INFINITY, l = 0.f;
    float o[2 * C::PPL];
#pragma unroll
    for (int i = 0; i < 2 * C::PPL; ++i) o[i] = 0.f;

    bool ok = true;
    for (int blk = b0; blk < b1; ++blk) {
      if (!mbar_wait(&full[stage], phase, p.status)) {
        ok = false;
        break;
      }
      const uint8_t* kt = smem + stage * C::STAGE_BYTES;
      const uint8_t* vt = kt + C::TILE_BYTES;
      float s[C::PASSES];
#pragma unroll
      for (int ps = 0; ps < C::PASSES; ++ps) {
        const int t = ps * C::TPP + tq;
        const uint4* krow = reinterpret_cast<const uint4*>(kt + ((t * HG + hh) * D + cq * 8) * 2);
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int c = 0; c < C::NCH; ++c) {
          const uint4 w = krow[c * C::LPT];
          acc0 = fmaf(qf[c * 8 + 0], bf16lo(w.x), acc0);
          acc1 = fmaf(qf[c * 8 + 1], bf16hi(w.x), acc1);
          acc0 = fmaf(qf[c * 8 + 2], bf16lo(w.y), acc0);
          acc1 = fmaf(qf[c * 8 + 3], bf16hi(w.y), acc1);
          acc0 = fmaf(qf[c * 8 + 4], bf16lo(w.z), acc0);
          acc1 = fmaf(qf[c * 8 + 5], bf16hi(w.z), acc1);
          acc0 = fmaf(qf[c * 8 + 6], bf16lo(w.w), acc0);
          acc1 = fmaf(qf[c * 8 + 7], bf16hi(w.w), acc1);
        }
        float acc = acc0 + acc1;
#pragma unroll
        for (int off = C::LPT / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        s[ps] = (blk * kBlock + t < n_cached) ? acc : -INFINITY;
      }
      float mb = s[0];
#pragma unroll
      for (int ps = 1; ps < C::PASSES; ++ps) mb = fmaxf(mb, s[ps]);
#pragma unroll
      for (int off = C::LPT; off < 32; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
      const float m_new = fmaxf(m, mb);
      const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m - m_new);
      float psum = 0.f;
#pragma unroll
      for (int ps = 0; ps < C::PASSES; ++ps) {
        s[ps] = (s[ps] == -INFINITY) ? 0.f : exp2f(s[ps] - m_new);
        psum += s[ps];
      }
#pragma unroll
      for (int off = C::LPT; off < 32; off <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      l = l * alpha + psum;
      m = m_new;
#pragma unroll
      for (int i = 0; i < 2 * C::PPL; ++i) o[i] *= alpha;
      const uint32_t* vrow = reinterpret_cast<const uint32_t*>(vt);
#pragma unroll
      for (int t = 0; t < kBlock; ++t) {
        const float pt = __shfl_sync(0xffffffffu, s[t / C::TPP], (t % C::TPP) * C::LPT);
#pragma unroll
        for (int i = 0; i < C::PPL; ++i) {
          const int j = lane + 32 * i;
          if (j < C::NPAIR) {
            const uint32_t w = vrow[(t * HG + hh) * C::NPAIR + j];
            o[2 * i] = fmaf(pt, bf16lo(w), o[2 * i]);
            o[2 * i + 1] = fmaf(pt, bf16hi(w), o[2 * i + 1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == C::NSTAGE) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (!ok) return;

    // The appended token: rotate k, fold it in from registers, write k/v to its cache row.
    if (p.append && split == nsplit - 1) {
      const __nv_bfloat16* krow = p.qkv + (int64_t)item * p.qkv_stride + p.k_col + (int64_t)head * D;
      const __nv_bfloat16* vsrc = p.qkv + (int64_t)item * p.qkv_stride + p.v_col + (int64_t)head * D;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < C::DPL; ++i) acc = fmaf(qf[i], load_rot<D>(p, krow, ((i / 8) * C::LPT + cq) * 8 + (i % 8), pos), acc);
#pragma unroll
      for (int off = C::LPT / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      const float m_new = fmaxf(m, acc);
      const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m - m_new);
      const float pn = exp2f(acc - m_new);
      l = l * alpha + pn;
      m = m_new;
      const uint32_t* v32 = reinterpret_cast<const uint32_t*>(vsrc);
#pragma unroll
      for (int i = 0; i < C::PPL; ++i) {
        const int j = lane + 32 * i;
        if (j < C::NPAIR) {
          const uint32_t w = v32[j];
          o[2 * i] = fmaf(pn, bf16lo(w), o[2 * i] * alpha);
          o[2 * i + 1] = fmaf(pn, bf16hi(w), o[2 * i + 1] * alpha);
        }
      }
      const int32_t* bt = p.block_table + (int64_t)p.item_slot[item] * p.bt_stride;
      const int64_t row = (int64_t)bt[pos / kBlock] * kBlock + pos % kBlock;
      if (row < 0 || row >= p.kv_rows) {
        if (lane == 0) set_error(p.status, CDB_ERR_INDEX);
      } else {
        const int64_t hstride = (int64_t)p.num_heads * D;
        __nv_bfloat16* kdst = p.kv + ((int64_t)(2 * p.cache_layer) * p.kv_rows + row) * hstride + (int64_t)head * D;
        __nv_bfloat16* vdst =
            p.kv + ((int64_t)(2 * p.cache_layer + 1) * p.kv_rows + row) * hstride + (int64_t)head * D;
        for (int d = lane; d < D; d += 32) {
          kdst[d] = f_to_bf16(load_rot<D>(p, krow, d, pos));
          vdst[d] = vsrc[d];
        }
      }
    }

    __nv_bfloat16* orow = p.out + (int64_t)item * p.out_stride + (int64_t)head * D;
    if (nsplit == 1) {
      const float inv = 1.f / l;
#pragma unroll
      for (int i = 0; i < C::PPL; ++i) {
        const int j = lane + 32 * i;
        if (j < C::NPAIR) reinterpret_cast<uint32_t*>(orow)[j] = pack_bf16x2(o[2 * i] * inv, o[2 * i + 1] * inv);
      }
      continue;
    }

    // Split-KV: publish the partial, the last CTA of this (row, head group) merges.
    const int64_t pidx = ((int64_t)item * p.num_heads + head) * kMaxSplits + split;
    float* po = p.part_o + pidx * D;
#pragma unroll
    for (int i = 0; i < C::PPL; ++i) {
      const int j = lane + 32 * i;
      if (j < C::NPAIR) {
        po[2 * j] = o[2 * i];
        po[2 * j + 1] = o[2 * i + 1];
      }
    }
    if (lane == 0) {
      p.part_ml[2 * pidx] = m;
      p.part_ml[2 * pidx + 1] = l;
    }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      int32_t* ctr = p.counters + (int64_t)item * p.num_heads + head;
      const int prev = atomicAdd(ctr, 1);
      last = (prev == nsplit - 1);
      if (last) atomicExch(ctr, 0);
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    __threadfence();
    const int64_t base = ((int64_t)item * p.num_heads + head) * kMaxSplits;
    float mx = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) mx = fmaxf(mx, __ldcg(p.part_ml + 2 * (base + sp)));
    float lsum = 0.f;
    float acc[2 * C::PPL];
#pragma unroll
    for (int i = 0; i < 2 * C::PPL; ++i) acc[i] = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float ms = __ldcg(p.part_ml + 2 * (base + sp));
      const float w = (ms == -INFINITY) ? 0.f : exp2f(ms - mx);
      lsum += w * __ldcg(p.part_ml + 2 * (base + sp) + 1);
      const float* ps = p.part_o + (base + sp) * D;
#pragma unroll
      for (int i = 0; i < C::PPL; ++i) {
        const int j = lane + 32 * i;
        if (j < C::NPAIR) {
          acc[2 * i] = fmaf(w, __ldcg(ps + 2 * j), acc[2 * i]);
          acc[2 * i + 1] = fmaf(w, __ldcg(ps + 2 * j + 1), acc[2 * i + 1]);
        }
      }
    }
    const float inv = 1.f / lsum;
#pragma unroll
    for (int i = 0; i < C::PPL; ++i) {
      const int j = lane + 32 * i;
      if (j < C::NPAIR) reinterpret_cast<uint32_t*>(orow)[j] = pack_bf16x2(acc[2 * i] * inv, acc[2 * i + 1] * inv);
    }
  }
}

// ------------------------------------------------------------------ work plan (one CTA)
__global__ void __launch_bounds__(1024) attn_plan_kernel(const int32_t* item_pos, int n, int append, int nhg,
                                                         int capacity, int scratch_items, int target_units,
                                                         int32_t* hdr, int4* units) {
  __shared__ int s_total, s_max, s_sb;
  __shared__ int s_warp[32];
  if (threadIdx.x == 0) {
    s_total = 0;
    s_max = 0;
  }
  __syncthreads();
  int local_total = 0, local_max = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int pos = item_pos[i];
    if (pos < 0) continue;
    const int nc = append ? pos : pos + 1;
    const int nb = (nc + kBlock - 1) / kBlock;
    local_total += nb;
    local_max = max(local_max, nb);
  }
  atomicAdd(&s_total, local_total);
  atomicMax(&s_max, local_max);
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long work = (long long)s_total * nhg;
    int sb = (int)((work + target_units - 1) / target_units);
    sb = max(sb, 4);
    sb = max(sb, (s_max + kMaxSplits - 1) / kMaxSplits);
    if (n > scratch_items) sb = max(sb, s_max);
    s_sb = max(sb, 1);
  }
  __syncthreads();
  const int sb = s_sb;
  // Exclusive scan of per-item unit counts, in chunks of blockDim.x items.
  int carry = 0;
  for (int start = 0; start < n; start += blockDim.x) {
    const int i = start + threadIdx.x;
    int cnt = 0, ns = 0;
    if (i < n) {
      const int pos = item_pos[i];
      if (pos >= 0) {
        const int nc = append ? pos : pos + 1;
        const int nb = (nc + kBlock - 1) / kBlock;
        ns = max(1, (nb + sb - 1) / sb);
        cnt = ns * nhg;
      }
    }
    // warp inclusive scan
    int v = cnt;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += t;
    }
    if (lane == 31) s_warp[w] = v;
    __syncthreads();
    if (w == 0) {
      int x = (lane < (int)(blockDim.x >> 5)) ? s_warp[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
      }
      s_warp[lane] = x;
    }
    __syncthreads();
    const int excl = carry + (w > 0 ? s_warp[w - 1] : 0) + v - cnt;
    if (i < n && cnt > 0) {
      for (int g = 0; g < nhg; ++g)
        for (int s = 0; s < ns; ++s) {
          const int idx = excl + g * ns + s;
          if (idx < capacity) units[idx] = make_int4(i, g, s, ns);
        }
    }
    const int chunk_total = s_warp[(blockDim.x >> 5) - 1];
    __syncthreads();
    carry += chunk_total;
  }
  if (threadIdx.x == 0) {
    hdr[0] = min(carry, capacity);
    hdr[1] = sb;
    hdr[2] = kMaxSplits;
    hdr[3] = 0;
  }
}

// ------------------------------------------------------------------ prefill rope + append
__global__ void rope_append_kernel(__nv_bfloat16* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col,
                                   __nv_bfloat16* kv, int64_t kv_rows, int cache_layer, const int32_t* block_table,
                                   int64_t bt_stride, const int32_t* item_slot, const int32_t* item_pos,
                                   int rope_mode, const void* rope_cos, const void* rope_sin, int n, int num_heads,
                                   int D) {
  const int item = blockIdx.x;
  const int pos = item_pos[item];
  if (pos < 0) return;
  const int head = blockIdx.y;
  __nv_bfloat16* q = qkv + (int64_t)item * qkv_stride + (int64_t)head * D;
  __nv_bfloat16* k = qkv + (int64_t)item * qkv_stride + k_col + (int64_t)head * D;
  const __nv_bfloat16* v = qkv + (int64_t)item * qkv_stride + v_col + (int64_t)head * D;
  float qr = 0.f, kr = 0.f;
  const int d = threadIdx.x;
  if (d < D) {
    if (rope_mode == 1) {
      const __nv_bfloat16* c = static_cast<const __nv_bfloat16*>(rope_cos) + (int64_t)pos * D;
      const __nv_bfloat16* s = static_cast<const __nv_bfloat16*>(rope_sin) + (int64_t)pos * D;
      qr = rope_elem(q, d, D, c, s);
      kr = rope_elem(k, d, D, c, s);
    } else if (rope_mode == 2) {
      const float* c = static_cast<const float*>(rope_cos) + (int64_t)pos * (D / 2);
      const float* s = static_cast<const float*>(rope_sin) + (int64_t)pos * (D / 2);
      qr = rope_elem_pairs(q, d, c, s);
      kr = rope_elem_pairs(k, d, c, s);
    } else {
      qr = bf16_to_f(q[d]);
      kr = bf16_to_f(k[d]);
    }
  }
  __syncthreads();
  if (d < D) {
    q[d] = f_to_bf16(qr);
    const int32_t* bt = block_table + (int64_t)item_slot[item] * bt_stride;
    const int64_t row = (int64_t)bt[pos / kBlock] * kBlock + pos % kBlock;
    const int64_t hstride = (int64_t)num_heads * D;
    kv[((int64_t)(2 * cache_layer) * kv_rows + row) * hstride + (int64_t)head * D + d] = f_to_bf16(kr);
    kv[((int64_t)(2 * cache_layer + 1) * kv_rows + row) * hstride + (int64_t)head * D + d] = v[d];
  }
}

// ------------------------------------------------------------------ tensor-map cache (host)
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

struct MapKey {
  const void* base;
  int layers;
  int64_t rows;
  int heads, d, hg;
  bool operator==(const MapKey& o) const {
    return base == o.base && layers == o.layers && rows == o.rows && heads == o.heads && d == o.d && hg == o.hg;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.base) ^ (std::hash<int64_t>()(k.rows) << 1) ^ ((size_t)k.layers << 7) ^
           ((size_t)k.heads << 17) ^ ((size_t)k.d << 27) ^ ((size_t)k.hg << 37);
  }
};

static int kv_tensor_map(CUtensorMap* out, const void* base, int layers, int64_t rows, int heads, int d, int hg) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{base, layers, rows, heads, d, hg};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return CDB_OK;
  }
  EncodeFn enc = get_encode();
  if (enc == nullptr) return CDB_ERR_TMA_ENCODE;
  const cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)heads, (cuuint64_t)rows, (cuuint64_t)(2 * layers)};
  const cuuint64_t strides[3] = {(cuuint64_t)d * 2, (cuuint64_t)heads * d * 2, (cuuint64_t)rows * heads * d * 2};
  const cuuint32_t box[4] = {(cuuint32_t)d, (cuuint32_t)hg, (cuuint32_t)kBlock, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return CDB_ERR_TMA_ENCODE;
  if (cache.size() > 64) cache.clear();
  cache.emplace(key, map);
  *out = map;
  return CDB_OK;
}

template <int D, int HG>
static int launch_attn(const CUtensorMap& map, const AttnParams& p, int num_ctas, cudaStream_t stream) {
  using C = AttnCfg<D, HG>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(decode_attn_kernel<D, HG>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return CDB_ERR_CUDA;
    attr_set = true;
  }
  decode_attn_kernel<D, HG><<<num_ctas, C::THREADS, C::SMEM, stream>>>(map, p);
  return cudaPeekAtLastError() == cudaSuccess ? CDB_OK : CDB_ERR_CUDA;
}

static int heads_per_cta(int num_heads, int head_dim) {
  if (head_dim == 128 && num_heads % 4 == 0) return 4;
  if (head_dim == 64 && num_heads % 4 == 0) return 4;
  if (head_dim == 96 && num_heads % 5 == 0) return 5;
  return 0;
}

}  // namespace cdb

using namespace cdb;

extern "C" int cdb_attn_plan(const int32_t* item_pos, int num_items, int append, int num_heads, int head_dim,
                             int block_size, int unit_capacity, int scratch_items, int num_sms, int32_t* plan_header,
                             void* units, void* stream) {
  if (block_size != kBlock || num_items < 0 || unit_capacity <= 0) return CDB_ERR_INVALID_ARGUMENT;
  const int hg = heads_per_cta(num_heads, head_dim);
  if (hg == 0) return CDB_ERR_UNSUPPORTED;
  const int target = 8 * (num_sms > 0 ? num_sms : 148);
  attn_plan_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(item_pos, num_items, append, num_heads / hg,
                                                                      unit_capacity, scratch_items, target,
                                                                      plan_header, static_cast<int4*>(units));
  return cudaPeekAtLastError() == cudaSuccess ? CDB_OK : CDB_ERR_CUDA;
}

extern "C" int64_t cdb_attn_scratch_bytes(int scratch_items, int num_heads, int head_dim) {
  const int64_t parts = (int64_t)scratch_items * num_heads * kMaxSplits;
  return parts * head_dim * 4 + parts * 2 * 4 + (int64_t)scratch_items * num_heads * 4;
}

extern "C" int cdb_paged_decode_attn_append(const void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col,
                                            void* out, int64_t out_stride, void* kv_base, int num_cache_layers,
                                            int64_t kv_rows, int cache_layer, const int32_t* block_table,
                                            int64_t block_table_stride, const int32_t* item_slot,
                                            const int32_t* item_pos, int rope_mode, const void* rope_cos,
                                            const void* rope_sin, int append, const int32_t* plan_header,
                                            const void* units, float* part_o, float* part_ml, int32_t* counters,
                                            int scratch_items, int num_items, int num_heads, int head_dim,
                                            int block_size, float scale, int num_ctas, int32_t* status,
                                            void* stream) {
  if (block_size != kBlock || cache_layer < 0 || cache_layer >= num_cache_layers || num_items < 0)
    return CDB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(kv_base) & 15) != 0 || (qkv_stride & 1) != 0) return CDB_ERR_INVALID_ARGUMENT;
  const int hg = heads_per_cta(num_heads, head_dim);
  if (hg == 0) return CDB_ERR_UNSUPPORTED;
  if (rope_mode < 0 || rope_mode > 2 || (rope_mode != 0 && (rope_cos == nullptr || rope_sin == nullptr)))
    return CDB_ERR_INVALID_ARGUMENT;
  (void)scratch_items;
  CUtensorMap map;
  const int rc = kv_tensor_map(&map, kv_base, num_cache_layers, kv_rows, num_heads, head_dim, hg);
  if (rc != CDB_OK) return rc;
  AttnParams p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.qkv_stride = qkv_stride;
  p.k_col = k_col;
  p.v_col = v_col;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.kv = static_cast<__nv_bfloat16*>(kv_base);
  p.kv_rows = kv_rows;
  p.cache_layer = cache_layer;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.item_slot = item_slot;
  p.item_pos = item_pos;
  p.rope_mode = rope_mode;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  p.append = append;
  p.hdr = plan_header;
  p.units = static_cast<const int4*>(units);
  p.part_o = part_o;
  p.part_ml = part_ml;
  p.counters = counters;
  p.num_heads = num_heads;
  p.scale_log2 = scale * kLog2e;
  p.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (num_ctas <= 0) num_ctas = 2 * 148;
  if (head_dim == 128) return launch_attn<128, 4>(map, p, num_ctas, st);
  if (head_dim == 64) return launch_attn<64, 4>(map, p, num_ctas, st);
  if (head_dim == 96) return launch_attn<96, 5>(map, p, num_ctas, st);
  return CDB_ERR_UNSUPPORTED;
}

extern "C" int cdb_rope_append_kv(void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col, void* kv_base,
                                  int num_cache_layers, int64_t kv_rows, int cache_layer, const int32_t* block_table,
                                  int64_t block_table_stride, const int32_t* item_slot, const int32_t* item_pos,
                                  int rope_mode, const void* rope_cos, const void* rope_sin, int num_items,
                                  int num_heads, int head_dim, int block_size, void* stream) {
  if (block_size != kBlock || cache_layer < 0 || cache_layer >= num_cache_layers || head_dim > 1024)
    return CDB_ERR_INVALID_ARGUMENT;
  if (num_items == 0) return CDB_OK;
  dim3 grid(num_items, num_heads);
  const int threads = ((head_dim + 31) / 32) * 32;
  rope_append_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(qkv), qkv_stride, k_col, v_col, static_cast<__nv_bfloat16*>(kv_base), kv_rows,
      cache_layer, block_table, block_table_stride, item_slot, item_pos, rope_mode, rope_cos, rope_sin, num_items,
      num_heads, head_dim);
  return cudaPeekAtLastError() == cudaSuccess ? CDB_OK : CDB_ERR_CUDA;
}
