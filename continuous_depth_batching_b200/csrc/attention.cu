// Ragged-depth paged decode attention for sm_100a.
//
// One launch serves one cache layer of a recurrent (or prefill) launch whose rows sit at
// different positions and recurrent steps. Work is split into units (row, head group,
// KV split) by cdb_attn_plan so CTAs see roughly equal byte counts despite ragged contexts.
//
// Decode rows first go through rope_append_kernel (rotate q in place, rotate k, write k/v to the
// row's cache slot), so the attention kernel itself only reads the cache: row p attends over
// positions [0, p]. Each CTA is warp specialised: one producer warp prefetches a unit's block
// ids with one coalesced load and streams its K and V pages through an NSTAGE-deep
// shared-memory ring with 4-D TMA tile loads (one 16-token x HG-head x D tile per page,
// completion on an mbarrier, no multicast); two consumer warps per head split every page's 16
// tokens, each keeping its own fp32 online-softmax state (QK dot products from conflict-free
// 16-byte shared-memory reads, base-2 softmax with warp shuffles, PV accumulation), and merge
// at the end of the unit. Splits of one (row, head) combine through scratch: the last warp to
// finish (atomic counter) merges the partial (m, l, o) triples and resets its counter.
#include <cuda.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "cdb_common.cuh"

namespace cdb {

constexpr int kMaxSplits = 64;
constexpr int kBlock = 16;           // tokens per page (block_size)
constexpr int kMaxPlanChunks = CDB_ATTN_PLAN_MAX_CHUNKS;
constexpr float kLog2e = 1.4426950408889634f;

template <int D, int HG>
struct AttnCfg {
  static constexpr int NSTAGE = 3;
  static constexpr int WPH = 2;                  // consumer warps per head
  static constexpr int TPW = kBlock / WPH;       // tokens of a page per warp
  static constexpr int LPT = (D == 96) ? 4 : 8;  // lanes cooperating on one token's QK dot
  static constexpr int DPL = D / LPT;            // dims per lane in QK
  static constexpr int TPP = 32 / LPT;           // tokens per pass
  static constexpr int PASSES = TPW / TPP;
  static constexpr int NPAIR = D / 2;
  static constexpr int PPL = (NPAIR + 31) / 32;  // bf16 pairs per lane in PV
  static constexpr int NCH = DPL / 8;            // 16-byte chunks per lane; lane cq owns chunks cq + c*LPT
  static constexpr int TILE_BYTES = kBlock * HG * D * 2;
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int CONSUMERS = HG * WPH;
  static constexpr int THREADS = (CONSUMERS + 1) * 32;
  static constexpr int MERGE_FLOATS = D + 2;
  static constexpr int SMEM = NSTAGE * STAGE_BYTES + 2 * NSTAGE * 8 + HG * MERGE_FLOATS * 4 + 64;
  static_assert(DPL % 8 == 0, "QK lane slice must be whole 16-byte chunks");
  static_assert(TPW % TPP == 0, "tokens per warp must be whole passes");
};

struct AttnParams {
  const __nv_bfloat16* qkv;
  int64_t qkv_stride;
  __nv_bfloat16* out;
  int64_t out_stride;
  int64_t kv_rows;
  int cache_layer;
  const int32_t* block_table;
  int64_t bt_stride;
  const int32_t* item_slot;
  const int32_t* item_pos;
  const int32_t* hdr;
  const int4* units;
  float* part_o;
  float* part_ml;
  int32_t* counters;
  int num_heads;
  float scale_log2;
  int32_t* status;
};

// A work unit: `row`'s head group `hg`, pages [b0, b1) of its cache, split `split` of `nsplit`.
struct Unit {
  int row, hg, split, nsplit, b0, b1;
};
__device__ __forceinline__ Unit decode_unit(int4 u) {
  return Unit{u.x, u.y >> 16, u.y & 0xffff, u.w, u.z >> 16, u.z & 0xffff};
}
// Units of chunk c: a range from the plan header, or unit c alone when segments are whole.
__device__ __forceinline__ void chunk_units(const int32_t* hdr, int c, int& u0, int& u1) {
  if (hdr[3]) {
    u0 = c;
    u1 = c + 1;
  } else {
    u0 = hdr[4 + c];
    u1 = hdr[5 + c];
  }
}

// Rotated value of element d of one head vector (Ouro split-half rotate_half RoPE with
// bf16 cos/sin, every product and the sum rounded to bf16 as PyTorch's bf16 ops round).
__device__ __forceinline__ float rope_half(float x_d, float x_partner, bool low_half, float c, float s) {
  const float rot = low_half ? -x_partner : x_partner;
  return round_bf16(round_bf16(x_d * c) + round_bf16(rot * s));
}

template <int D, int HG>
__global__ void __launch_bounds__(AttnCfg<D, HG>::THREADS) decode_attn_kernel(const __grid_constant__ CUtensorMap map,
                                                                              AttnParams p) {
  using C = AttnCfg<D, HG>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NSTAGE * C::STAGE_BYTES);
  uint64_t* empty = full + C::NSTAGE;
  float* merge = reinterpret_cast<float*>(empty + C::NSTAGE);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::CONSUMERS);
    }
    fence_barrier_init();
  }
  if (warp == C::CONSUMERS && lane == 0) prefetch_tensormap(&map);
  __syncthreads();
  pdl_trigger();
  pdl_wait();

  const int n_chunks = p.hdr[1];

  if (warp == C::CONSUMERS) {
    // ------------------------------------------------------------- producer warp
    if (lane == 0) prefetch_tensormap(&map);
    int stage = 0;
    uint32_t phase = 0;
    bool alive = true;
    for (int c = blockIdx.x; c < n_chunks && alive; c += gridDim.x) {
    int u0, u1;
    chunk_units(p.hdr, c, u0, u1);
    for (int u = u0; u < u1 && alive; ++u) {
      const Unit unit = decode_unit(p.units[u]);
      const int b0 = unit.b0;
      const int b1 = unit.b1;
      const int32_t* bt = p.block_table + (int64_t)p.item_slot[unit.row] * p.bt_stride;
      for (int base = b0; base < b1 && alive; base += 32) {
        const int my = base + lane < b1 ? bt[base + lane] : 0;
        const int cnt = min(32, b1 - base);
        for (int i = 0; i < cnt; ++i) {
          const int block_id = __shfl_sync(0xffffffffu, my, i);
          if (lane == 0) {
            if (mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
              mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
              uint8_t* dst = smem + stage * C::STAGE_BYTES;
              tma_load_4d(dst, &map, &full[stage], 0, unit.hg * HG, block_id * kBlock, 2 * p.cache_layer);
              tma_load_4d(dst + C::TILE_BYTES, &map, &full[stage], 0, unit.hg * HG, block_id * kBlock,
                          2 * p.cache_layer + 1);
            } else {
              alive = false;
            }
          }
          alive = __shfl_sync(0xffffffffu, alive, 0);
          if (!alive) break;
          if (++stage == C::NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    }
    return;
  }

  // --------------------------------------------------------------- consumer warps
  const int hh = warp / C::WPH;   // head within the group
  const int sub = warp % C::WPH;  // which half of every page's tokens
  const int tq = lane / C::LPT;   // token slot within a pass
  const int cq = lane % C::LPT;   // dim slice within the token
  float* mslot = merge + hh * C::MERGE_FLOATS;
  const int bar_id = 1 + hh;
  int stage = 0;
  uint32_t phase = 0;
  bool alive = true;

  for (int c = blockIdx.x; c < n_chunks; c += gridDim.x) {
  int u0, u1;
  chunk_units(p.hdr, c, u0, u1);
  for (int u = u0; u < u1; ++u) {
    const Unit unit = decode_unit(p.units[u]);
    const int item = unit.row;
    const int head = unit.hg * HG + hh;
    const int split = unit.split;
    const int nsplit = unit.nsplit;
    const int pos = p.item_pos[item];
    const int n_cached = pos + 1;
    const int b0 = unit.b0;
    const int b1 = unit.b1;

    // this lane's q slice (already rotated), pre-scaled by softmax_scale*log2(e)
    const __nv_bfloat16* qrow = p.qkv + (int64_t)item * p.qkv_stride + (int64_t)head * D;
    float qf[C::DPL];
#pragma unroll
    for (int c = 0; c < C::NCH; ++c) {
      const uint4 w = *reinterpret_cast<const uint4*>(qrow + (c * C::LPT + cq) * 8);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        qf[c * 8 + 2 * k] = bf16lo(ws[k]) * p.scale_log2;
        qf[c * 8 + 2 * k + 1] = bf16hi(ws[k]) * p.scale_log2;
      }
    }

    float m = -INFINITY, l = 0.f;
    float o[2 * C::PPL];
#pragma unroll
    for (int i = 0; i < 2 * C::PPL; ++i) o[i] = 0.f;

    for (int blk = b0; blk < b1; ++blk) {
      if (alive && !mbar_wait(&full[stage], phase, p.status)) alive = false;
      if (alive) {
        const uint8_t* kt = smem + stage * C::STAGE_BYTES;
        const uint8_t* vt = kt + C::TILE_BYTES;
        float s[C::PASSES];
#pragma unroll
        for (int ps = 0; ps < C::PASSES; ++ps) {
          const int t = sub * C::TPW + ps * C::TPP + tq;
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
        for (int tt = 0; tt < C::TPW; ++tt) {
          const int t = sub * C::TPW + tt;
          const float pt = __shfl_sync(0xffffffffu, s[tt / C::TPP], (tt % C::TPP) * C::LPT);
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
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == C::NSTAGE) {
        stage = 0;
        phase ^= 1u;
      }
    }

    // merge the two token halves of this head
    if (sub == 1) {
#pragma unroll
      for (int i = 0; i < C::PPL; ++i) {
        const int j = lane + 32 * i;
        if (j < C::NPAIR) {
          mslot[2 * j] = o[2 * i];
          mslot[2 * j + 1] = o[2 * i + 1];
        }
      }
      if (lane == 0) {
        mslot[D] = m;
        mslot[D + 1] = l;
      }
    }
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(64) : "memory");
    if (sub == 0) {
      const float m2 = mslot[D], l2 = mslot[D + 1];
      const float mm = fmaxf(m, m2);
      const float w1 = (m == -INFINITY) ? 0.f : exp2f(m - mm);
      const float w2 = (m2 == -INFINITY) ? 0.f : exp2f(m2 - mm);
      l = l * w1 + l2 * w2;
      m = mm;
#pragma unroll
      for (int i = 0; i < C::PPL; ++i) {
        const int j = lane + 32 * i;
        if (j < C::NPAIR) {
          o[2 * i] = o[2 * i] * w1 + mslot[2 * j] * w2;
          o[2 * i + 1] = o[2 * i + 1] * w1 + mslot[2 * j + 1] * w2;
        }
      }
    }
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(64) : "memory");
    if (sub != 0 || !alive) continue;

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

    // Split-KV: publish the partial; the last warp of this (row, head) merges all splits.
    const int64_t pidx = ((int64_t)item * p.num_heads + head) * kMaxSplits + split;
    float* po = p.part_o + pidx * D;
#pragma unroll
    for (int i = 0; i < C::PPL; ++i) {
      const int j = lane + 32 * i;
      if (j < C::NPAIR) *reinterpret_cast<float2*>(po + 2 * j) = make_float2(o[2 * i], o[2 * i + 1]);
    }
    if (lane == 0) *reinterpret_cast<float2*>(p.part_ml + 2 * pidx) = make_float2(m, l);
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      __threadfence();
      int32_t* ctr = p.counters + (int64_t)item * p.num_heads + head;
      const int prev = atomicAdd(ctr, 1);
      last = (prev == nsplit - 1);
      if (last) {
        atomicExch(ctr, 0);
        __threadfence();
      }
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    const int64_t base = ((int64_t)item * p.num_heads + head) * kMaxSplits;
    float mx = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) mx = fmaxf(mx, __ldcg(p.part_ml + 2 * (base + sp)));
    float lsum = 0.f;
    float acc[2 * C::PPL];
#pragma unroll
    for (int i = 0; i < 2 * C::PPL; ++i) acc[i] = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml + 2 * (base + sp)));
      const float w = (ml.x == -INFINITY) ? 0.f : exp2f(ml.x - mx);
      lsum += w * ml.y;
      const float* ps = p.part_o + (base + sp) * D;
#pragma unroll
      for (int i = 0; i < C::PPL; ++i) {
        const int j = lane + 32 * i;
        if (j < C::NPAIR) {
          const float2 v = __ldcg(reinterpret_cast<const float2*>(ps + 2 * j));
          acc[2 * i] = fmaf(w, v.x, acc[2 * i]);
          acc[2 * i + 1] = fmaf(w, v.y, acc[2 * i + 1]);
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
}

// ------------------------------------------------------------------ work plan (one CTA)
// Exclusive block-wide scan of one int per thread (blockDim.x == 1024); `total` gets the sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += t;
  }
  if (lane == 31) s_warp[w] = x;
  __syncthreads();
  if (w == 0) {
    int y = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, y, o);
      if (lane >= o) y += t;
    }
    s_warp[lane] = y;
  }
  __syncthreads();
  const int excl = (w > 0 ? s_warp[w - 1] : 0) + x - v;
  total = s_warp[31];
  __syncthreads();
  return excl;
}

// Balanced plan. The launch's work is the sequence of pages of every (row, head group) segment,
// rows in order and head groups inner, cut into n_chunks equal chunks of `ch` pages (about one
// chunk per CTA). A segment crossing chunk boundaries becomes one unit per chunk it touches
// (split-KV pieces, merged by the last warp to finish); chunk c's units are
// [hdr[4 + c], hdr[5 + c]). Every CTA streams the same number of pages, so no CTA is left with
// a whole extra segment at the end. When the rows exceed the split-combine scratch
// (n > scratch_items) segments are not split: one unit each, dealt round-robin (hdr[3] = 1).
// Units: int4 {row, head_group << 16 | split, first_page << 16 | end_page, num_splits}.
__global__ void __launch_bounds__(1024) attn_plan_kernel(const int32_t* item_pos, int n, int nhg, int capacity,
                                                         int scratch_items, int target_chunks, int32_t* hdr,
                                                         int4* units) {
  __shared__ int s_total, s_max, s_ch, s_nch;
  __shared__ int s_warp[32];
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) {
    s_total = 0;
    s_max = 0;
  }
  __syncthreads();
  int local_total = 0, local_max = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int pos = item_pos[i];
    if (pos < 0) continue;
    const int nb = (pos + kBlock) / kBlock;  // pages of the cached positions 0..pos
    local_total += nb;
    local_max = max(local_max, nb);
  }
  atomicAdd(&s_total, local_total);
  atomicMax(&s_max, local_max);
  __syncthreads();
  const bool whole = n > scratch_items;
  if (threadIdx.x == 0) {
    const long long T = (long long)s_total * nhg;
    const int C = max(1, min(target_chunks, kMaxPlanChunks));
    long long ch = (T + C - 1) / C;
    ch = max(ch, (long long)((s_max + kMaxSplits - 3) / (kMaxSplits - 2)));  // <= kMaxSplits pieces a segment
    ch = max(ch, 2LL);
    s_ch = (int)ch;
    s_nch = T > 0 ? (int)((T + ch - 1) / ch) : 0;
  }
  __syncthreads();
  const long long ch = s_ch;
  const int nch = s_nch;
  int carry_p = 0, carry_u = 0;
  for (int start = 0; start < n; start += blockDim.x) {
    const int i = start + threadIdx.x;
    int p = 0;
    if (i < n) {
      const int pos = item_pos[i];
      if (pos >= 0) p = (pos + kBlock) / kBlock;
    }
    int tile_pages;
    const int ep = block_exclusive_scan(p, s_warp, tile_pages);
    const long long S0 = (long long)(carry_p + ep) * nhg;  // first page of segment (i, 0)
    int pieces = 0;
    if (p > 0) {
      if (whole) {
        pieces = nhg;
      } else {
        for (int g = 0; g < nhg; ++g) {
          const long long S = S0 + (long long)g * p;
          pieces += (int)((S + p - 1) / ch - S / ch + 1);
        }
      }
    }
    int tile_units;
    int u = carry_u + block_exclusive_scan(pieces, s_warp, tile_units);
    if (p > 0) {
      for (int g = 0; g < nhg; ++g) {
        if (whole) {
          if (u < capacity) units[u] = make_int4(i, g << 16, p, 1);
          ++u;
          continue;
        }
        const long long S = S0 + (long long)g * p;
        const long long fc = S / ch;
        const int ns = (int)((S + p - 1) / ch - fc + 1);
        for (int k = 0; k < ns; ++k) {
          const long long c = fc + k;
          const int b0 = (int)max(0LL, c * ch - S);
          const int b1 = (int)min((long long)p, (c + 1) * ch - S);
          if (u < capacity) units[u] = make_int4(i, (g << 16) | k, (b0 << 16) | b1, ns);
          if (c * ch >= S && c < nch) hdr[4 + c] = min(u, capacity);  // chunk c starts in this segment
          ++u;
        }
      }
    }
    carry_p += tile_pages;
    carry_u += tile_units;
  }
  if (threadIdx.x == 0) {
    const int n_units = min(carry_u, capacity);
    hdr[0] = n_units;
    hdr[1] = whole ? n_units : nch;
    hdr[2] = kMaxSplits;
    hdr[3] = whole ? 1 : 0;
    if (!whole) hdr[4 + nch] = n_units;
  }
}

// ------------------------------------------------------------------ rope + append
// One CTA per row: rotate q in place, rotate k, write k and v to the row's cache slot. Each
// thread owns one rotation pair of one head, so the in-place update needs no synchronisation.
// qk_bias (bf16 [2][heads][D], q bias then k bias; may be null) is added to q and k in bf16
// before the rotation (HuginnAttention.forward, modeling_huginn.py:261-264).
__global__ void rope_append_kernel(__nv_bfloat16* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col,
                                   __nv_bfloat16* kv, int64_t kv_rows, int cache_layer, const int32_t* block_table,
                                   int64_t bt_stride, const int32_t* item_slot, const int32_t* item_pos,
                                   int rope_mode, const void* rope_cos, const void* rope_sin,
                                   const __nv_bfloat16* qk_bias, int num_heads, int D, int32_t* status) {
  pdl_trigger();
  pdl_wait();
  const int item = blockIdx.x;
  const int pos = item_pos[item];
  if (pos < 0) return;
  const int32_t* bt = block_table + (int64_t)item_slot[item] * bt_stride;
  const int blk = bt[pos / kBlock];
  const int64_t row = (int64_t)blk * kBlock + pos % kBlock;
  if (blk < 0 || row >= kv_rows) {
    if (threadIdx.x == 0) set_error(status, CDB_ERR_INDEX);
    return;
  }
  const int64_t hstride = (int64_t)num_heads * D;
  __nv_bfloat16* q = qkv + (int64_t)item * qkv_stride;
  const __nv_bfloat16* k = q + k_col;
  const __nv_bfloat16* v = q + v_col;
  __nv_bfloat16* kd = kv + ((int64_t)(2 * cache_layer) * kv_rows + row) * hstride;
  __nv_bfloat16* vd = kv + ((int64_t)(2 * cache_layer + 1) * kv_rows + row) * hstride;
  const int half = D / 2;
  const __nv_bfloat16* kb = qk_bias ? qk_bias + (int64_t)num_heads * D : nullptr;
  // element d of head h of q (or k), with the bias added in bf16 when present
  auto qval = [&](int64_t hb, int d) {
    const float x = bf16_to_f(q[hb + d]);
    return qk_bias ? round_bf16(x + bf16_to_f(qk_bias[hb + d])) : x;
  };
  auto kval = [&](int64_t hb, int d) {
    const float x = bf16_to_f(k[hb + d]);
    return kb ? round_bf16(x + bf16_to_f(kb[hb + d])) : x;
  };
  for (int i = threadIdx.x; i < num_heads * half; i += blockDim.x) {
    const int h = i / half, j = i % half;
    const int64_t hb = (int64_t)h * D;
    if (rope_mode == 1) {
      const __nv_bfloat16* cr = static_cast<const __nv_bfloat16*>(rope_cos) + (int64_t)pos * D;
      const __nv_bfloat16* sr = static_cast<const __nv_bfloat16*>(rope_sin) + (int64_t)pos * D;
      const int d0 = j, d1 = j + half;
      const float q0 = qval(hb, d0), q1 = qval(hb, d1);
      const float k0 = kval(hb, d0), k1 = kval(hb, d1);
      const float c0 = bf16_to_f(cr[d0]), s0 = bf16_to_f(sr[d0]), c1 = bf16_to_f(cr[d1]), s1 = bf16_to_f(sr[d1]);
      q[hb + d0] = f_to_bf16(rope_half(q0, q1, true, c0, s0));
      q[hb + d1] = f_to_bf16(rope_half(q1, q0, false, c1, s1));
      kd[hb + d0] = f_to_bf16(rope_half(k0, k1, true, c0, s0));
      kd[hb + d1] = f_to_bf16(rope_half(k1, k0, false, c1, s1));
      vd[hb + d0] = v[hb + d0];
      vd[hb + d1] = v[hb + d1];
    } else if (rope_mode == 2) {
      // Huginn interleaved pairs (2j, 2j+1) rotated in fp32 (modeling_huginn.py:178-196).
      const float* cr = static_cast<const float*>(rope_cos) + (int64_t)pos * half;
      const float* sr = static_cast<const float*>(rope_sin) + (int64_t)pos * half;
      // Each product and the sum rounded separately (no contraction), as the fp32 tensor ops do.
      const int d0 = 2 * j, d1 = 2 * j + 1;
      const float c = cr[j], s = sr[j];
      const float q0 = qval(hb, d0), q1 = qval(hb, d1);
      const float k0 = kval(hb, d0), k1 = kval(hb, d1);
      q[hb + d0] = f_to_bf16(__fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, s)));
      q[hb + d1] = f_to_bf16(__fadd_rn(__fmul_rn(q1, c), __fmul_rn(q0, s)));
      kd[hb + d0] = f_to_bf16(__fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, s)));
      kd[hb + d1] = f_to_bf16(__fadd_rn(__fmul_rn(k1, c), __fmul_rn(k0, s)));
      vd[hb + d0] = v[hb + d0];
      vd[hb + d1] = v[hb + d1];
    } else {
      const int d0 = 2 * j, d1 = 2 * j + 1;
      if (qk_bias) {
        q[hb + d0] = f_to_bf16(qval(hb, d0));
        q[hb + d1] = f_to_bf16(qval(hb, d1));
      }
      kd[hb + d0] = f_to_bf16(kval(hb, d0));
      kd[hb + d1] = f_to_bf16(kval(hb, d1));
      vd[hb + d0] = v[hb + d0];
      vd[hb + d1] = v[hb + d1];
    }
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
  return launch_pdl(decode_attn_kernel<D, HG>, dim3(num_ctas), dim3(C::THREADS), C::SMEM, stream, map, p) ==
                 cudaSuccess
             ? CDB_OK
             : CDB_ERR_CUDA;
}

static int heads_per_cta(int num_heads, int head_dim) {
  if (head_dim == 128 && num_heads % 4 == 0) return 4;
  if (head_dim == 64 && num_heads % 4 == 0) return 4;
  if (head_dim == 96 && num_heads % 5 == 0) return 5;
  return 0;
}

static int launch_rope_append(void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col, void* kv_base,
                              int64_t kv_rows, int cache_layer, const int32_t* block_table, int64_t bt_stride,
                              const int32_t* item_slot, const int32_t* item_pos, int rope_mode, const void* rope_cos,
                              const void* rope_sin, const void* qk_bias, int num_items, int num_heads, int head_dim,
                              int32_t* status, cudaStream_t st) {
  if (num_items == 0) return CDB_OK;
  const int pairs = num_heads * (head_dim / 2);
  const int threads = pairs >= 1024 ? 1024 : ((pairs + 31) / 32) * 32;
  return launch_pdl(rope_append_kernel, dim3(num_items), dim3(threads), 0, st, static_cast<__nv_bfloat16*>(qkv),
                    qkv_stride, k_col, v_col, static_cast<__nv_bfloat16*>(kv_base), kv_rows, cache_layer, block_table,
                    bt_stride, item_slot, item_pos, rope_mode, rope_cos, rope_sin,
                    static_cast<const __nv_bfloat16*>(qk_bias), num_heads, head_dim, status) == cudaSuccess
             ? CDB_OK
             : CDB_ERR_CUDA;
}

}  // namespace cdb

using namespace cdb;

extern "C" int cdb_attn_plan(const int32_t* item_pos, int num_items, int append, int num_heads, int head_dim,
                             int block_size, int unit_capacity, int scratch_items, int num_sms, int32_t* plan_header,
                             void* units, void* stream) {
  if (block_size != kBlock || num_items < 0 || unit_capacity <= 0) return CDB_ERR_INVALID_ARGUMENT;
  const int hg = heads_per_cta(num_heads, head_dim);
  if (hg == 0) return CDB_ERR_UNSUPPORTED;
  (void)append;  // the attention kernel reads only cached rows; append happens before it
  // one chunk per attention CTA: the decode launch runs 2 CTAs per SM
  const int target = 2 * (num_sms > 0 ? num_sms : 148);
  return launch_pdl(attn_plan_kernel, dim3(1), dim3(1024), 0, static_cast<cudaStream_t>(stream), item_pos, num_items,
                    num_heads / hg, unit_capacity, scratch_items, target, plan_header,
                    static_cast<int4*>(units)) == cudaSuccess
             ? CDB_OK
             : CDB_ERR_CUDA;
}

extern "C" int64_t cdb_attn_scratch_bytes(int scratch_items, int num_heads, int head_dim) {
  const int64_t parts = (int64_t)scratch_items * num_heads * kMaxSplits;
  return parts * head_dim * 4 + parts * 2 * 4 + (int64_t)scratch_items * num_heads * 4;
}

extern "C" int cdb_paged_decode_attn_append(void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col, void* out,
                                            int64_t out_stride, void* kv_base, int num_cache_layers, int64_t kv_rows,
                                            int cache_layer, const int32_t* block_table, int64_t block_table_stride,
                                            const int32_t* item_slot, const int32_t* item_pos, int rope_mode,
                                            const void* rope_cos, const void* rope_sin, const void* qk_bias,
                                            int append, const int32_t* plan_header, const void* units, float* part_o,
                                            float* part_ml, int32_t* counters, int scratch_items, int num_items,
                                            int num_heads, int head_dim, int block_size, float scale, int num_ctas,
                                            int32_t* status, void* stream) {
  if (block_size != kBlock || cache_layer < 0 || cache_layer >= num_cache_layers || num_items < 0)
    return CDB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(kv_base) & 15) || (reinterpret_cast<uintptr_t>(qkv) & 15) || (qkv_stride & 7) ||
      (k_col & 7) || (v_col & 7) || (out_stride & 1))
    return CDB_ERR_INVALID_ARGUMENT;
  const int hg = heads_per_cta(num_heads, head_dim);
  if (hg == 0) return CDB_ERR_UNSUPPORTED;
  if (rope_mode < 0 || rope_mode > 2 || (append && rope_mode != 0 && (rope_cos == nullptr || rope_sin == nullptr)))
    return CDB_ERR_INVALID_ARGUMENT;
  (void)scratch_items;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (append) {
    const int rc = launch_rope_append(qkv, qkv_stride, k_col, v_col, kv_base, kv_rows, cache_layer, block_table,
                                      block_table_stride, item_slot, item_pos, rope_mode, rope_cos, rope_sin, qk_bias,
                                      num_items, num_heads, head_dim, status, st);
    if (rc != CDB_OK) return rc;
  }
  CUtensorMap map;
  const int rc = kv_tensor_map(&map, kv_base, num_cache_layers, kv_rows, num_heads, head_dim, hg);
  if (rc != CDB_OK) return rc;
  AttnParams p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.qkv_stride = qkv_stride;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.kv_rows = kv_rows;
  p.cache_layer = cache_layer;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.item_slot = item_slot;
  p.item_pos = item_pos;
  p.hdr = plan_header;
  p.units = static_cast<const int4*>(units);
  p.part_o = part_o;
  p.part_ml = part_ml;
  p.counters = counters;
  p.num_heads = num_heads;
  p.scale_log2 = scale * kLog2e;
  p.status = status;
  if (num_ctas <= 0) num_ctas = 2 * 148;
  if (head_dim == 128) return launch_attn<128, 4>(map, p, num_ctas, st);
  if (head_dim == 64) return launch_attn<64, 4>(map, p, num_ctas, st);
  if (head_dim == 96) return launch_attn<96, 5>(map, p, num_ctas, st);
  return CDB_ERR_UNSUPPORTED;
}

extern "C" int cdb_rope_append_kv(void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col, void* kv_base,
                                  int num_cache_layers, int64_t kv_rows, int cache_layer, const int32_t* block_table,
                                  int64_t block_table_stride, const int32_t* item_slot, const int32_t* item_pos,
                                  int rope_mode, const void* rope_cos, const void* rope_sin, const void* qk_bias,
                                  int num_items, int num_heads, int head_dim, int block_size, void* stream) {
  if (block_size != kBlock || cache_layer < 0 || cache_layer >= num_cache_layers || head_dim % 2 != 0 ||
      rope_mode < 0 || rope_mode > 2)
    return CDB_ERR_INVALID_ARGUMENT;
  return launch_rope_append(qkv, qkv_stride, k_col, v_col, kv_base, kv_rows, cache_layer, block_table,
                            block_table_stride, item_slot, item_pos, rope_mode, rope_cos, rope_sin, qk_bias, num_items,
                            num_heads, head_dim, nullptr, static_cast<cudaStream_t>(stream));
}

// ======================================================================================
// Allocation-free variant of cdb_paged_decode_attn_append.
//
// Some callers cannot call cudaMalloc at all: a function registered as the model's attention
// hook runs inside the host framework's CUDA-graph capture (allocation is not permitted while a
// stream is being captured), and a plugin that is handed only tensors has no allocator to ask.
// For them the work plan and the split-KV combine scratch of this entry point live in one
// file-scope device array instead of caller buffers. Every GPU that loads the library holds the
// array (4,788,992 bytes) until the process exits.
// ======================================================================================
namespace cdb {
namespace noalloc {
constexpr int kRowHeads = 128;    // (rows x heads) the split-combine scratch covers
constexpr int kMaxUnits = 32768;  // work-plan capacity (units of row x head group x split)
constexpr int kMaxHeadDim = 128;
constexpr size_t kPartOFloats = (size_t)kRowHeads * kMaxSplits * kMaxHeadDim;
constexpr size_t kPartMLFloats = (size_t)kRowHeads * kMaxSplits * 2;
constexpr size_t kOffPartML = kPartOFloats * 4;
constexpr size_t kOffCounters = kOffPartML + kPartMLFloats * 4;
constexpr size_t kOffHeader = kOffCounters + (size_t)kRowHeads * 4;
constexpr size_t kOffUnits = (kOffHeader + CDB_ATTN_PLAN_HEADER_INTS * 4 + 255) / 256 * 256;
constexpr size_t kBytes = kOffUnits + (size_t)kMaxUnits * 16;
constexpr int kMaxDevices = 64;
}  // namespace noalloc
}  // namespace cdb

// The scratch itself. Host code must not use this name as a device address: it resolves to a
// host-side shadow. Its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t cdb_noalloc_scratch[cdb::noalloc::kBytes];

namespace cdb {
namespace noalloc {

// Device address of the scratch array on the current device, looked up once per device with
// that device current (the first call on a device does this; make it before any stream capture).
static int scratch_address(uint8_t** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CDB_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, cdb_noalloc_scratch) != cudaSuccess || p == nullptr) return CDB_ERR_CUDA;
    addr[dev] = p;
  }
  *out = static_cast<uint8_t*>(addr[dev]);
  return CDB_OK;
}

// The KV pool tensor map, encoded on the stack (the cached path keeps a host-side table).
static int encode_kv_map(CUtensorMap* map, const void* base, int layers, int64_t rows, int heads, int d, int hg) {
  EncodeFn enc = get_encode();
  if (enc == nullptr) return CDB_ERR_TMA_ENCODE;
  const cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)heads, (cuuint64_t)rows, (cuuint64_t)(2 * layers)};
  const cuuint64_t strides[3] = {(cuuint64_t)d * 2, (cuuint64_t)heads * d * 2, (cuuint64_t)rows * heads * d * 2};
  const cuuint32_t box[4] = {(cuuint32_t)d, (cuuint32_t)hg, (cuuint32_t)kBlock, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  std::memset(map, 0, sizeof(*map));
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? CDB_OK
             : CDB_ERR_TMA_ENCODE;
}

}  // namespace noalloc
}  // namespace cdb

extern "C" int cdb_paged_decode_attn_append_static(void* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col,
                                                   void* out, int64_t out_stride, void* kv_base, int num_cache_layers,
                                                   int64_t kv_rows, int cache_layer, const int32_t* block_table,
                                                   int64_t block_table_stride, const int32_t* item_slot,
                                                   const int32_t* item_pos, int rope_mode, const void* rope_cos,
                                                   const void* rope_sin, const void* qk_bias, int append,
                                                   int num_items, int num_heads,
                                                   int head_dim, int block_size, float scale, int num_ctas,
                                                   int32_t* status, void* stream) {
  using namespace cdb::noalloc;
  if (block_size != kBlock || cache_layer < 0 || cache_layer >= num_cache_layers || num_items < 0)
    return CDB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(kv_base) & 15) || (reinterpret_cast<uintptr_t>(qkv) & 15) || (qkv_stride & 7) ||
      (k_col & 7) || (v_col & 7) || (out_stride & 1))
    return CDB_ERR_INVALID_ARGUMENT;
  const int hg = heads_per_cta(num_heads, head_dim);
  if (hg == 0) return CDB_ERR_UNSUPPORTED;
  if (rope_mode < 0 || rope_mode > 2 || (append && rope_mode != 0 && (rope_cos == nullptr || rope_sin == nullptr)))
    return CDB_ERR_INVALID_ARGUMENT;
  // Limits of the static scratch: head_dim <= 128, num_heads <= 128, and the work plan of an
  // unsplit launch (num_items x num_heads/heads_per_CTA units) within kMaxUnits.
  const int scratch_items = kRowHeads / num_heads;
  if (head_dim > kMaxHeadDim || scratch_items < 1 || (int64_t)num_items * (num_heads / hg) > kMaxUnits)
    return CDB_ERR_SCRATCH_LIMIT;
  uint8_t* base = nullptr;
  int rc = scratch_address(&base);
  if (rc != CDB_OK) return rc;
  if (num_items == 0) return CDB_OK;
  float* part_o = reinterpret_cast<float*>(base);
  float* part_ml = reinterpret_cast<float*>(base + kOffPartML);
  int32_t* counters = reinterpret_cast<int32_t*>(base + kOffCounters);
  int32_t* header = reinterpret_cast<int32_t*>(base + kOffHeader);
  void* units = base + kOffUnits;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: the split counters must start at zero.
  if (cudaMemsetAsync(counters, 0, (size_t)kRowHeads * 4, st) != cudaSuccess) return CDB_ERR_CUDA;
  if (append) {
    rc = launch_rope_append(qkv, qkv_stride, k_col, v_col, kv_base, kv_rows, cache_layer, block_table,
                            block_table_stride, item_slot, item_pos, rope_mode, rope_cos, rope_sin, qk_bias,
                            num_items, num_heads, head_dim, status, st);
    if (rc != CDB_OK) return rc;
  }
  if (num_ctas <= 0) num_ctas = 2 * 148;
  if (launch_pdl(attn_plan_kernel, dim3(1), dim3(1024), 0, st, item_pos, num_items, num_heads / hg, kMaxUnits,
                 scratch_items, num_ctas, header, static_cast<int4*>(units)) != cudaSuccess)
    return CDB_ERR_CUDA;
  CUtensorMap map;
  rc = encode_kv_map(&map, kv_base, num_cache_layers, kv_rows, num_heads, head_dim, hg);
  if (rc != CDB_OK) return rc;
  AttnParams p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.qkv_stride = qkv_stride;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.kv_rows = kv_rows;
  p.cache_layer = cache_layer;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.item_slot = item_slot;
  p.item_pos = item_pos;
  p.hdr = header;
  p.units = static_cast<const int4*>(units);
  p.part_o = part_o;
  p.part_ml = part_ml;
  p.counters = counters;
  p.num_heads = num_heads;
  p.scale_log2 = scale * kLog2e;
  p.status = status;
  if (num_ctas <= 0) num_ctas = 2 * 148;
  if (head_dim == 128) return launch_attn<128, 4>(map, p, num_ctas, st);
  if (head_dim == 64) return launch_attn<64, 4>(map, p, num_ctas, st);
  if (head_dim == 96) return launch_attn<96, 5>(map, p, num_ctas, st);
  return CDB_ERR_UNSUPPORTED;
}
