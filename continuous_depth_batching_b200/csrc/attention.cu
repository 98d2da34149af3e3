// Ragged-depth paged decode attention for sm_100a.
//
// One launch serves one cache layer of a recurrent (or prefill) launch whose rows sit at
// different positions and recurrent steps. Work is split into units (row, head group,
// KV split) by cdb_attn_plan so CTAs see roughly equal byte counts despite ragged contexts.
//
// The new token of each row is appended in one of two ways. append == 1: rope_append_kernel
// first rotates q in place, rotates k and writes k/v to the row's cache slot, and the attention
// kernel then only reads the cache. append == 2 (fused, one launch): the attention kernel rotates
// q in registers, and the warp that reads position p of a row's last staged page computes the
// rotated k and v itself, writes them to the cache and uses them for position p from registers
// (the bytes TMA staged for that row are not used). Either way row p attends over [0, p].
// Each CTA is warp specialised: one producer warp prefetches a unit's block
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
  static constexpr int SMEM = NSTAGE * STAGE_BYTES + 3 * NSTAGE * 8 + HG * MERGE_FLOATS * 4 + 64;
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
  int num_items;  // rows of item_slot / item_pos
  float scale_log2;
  int32_t* status;
  // Fused append (append == 2): q is read unrotated and rotated in registers; the warp that
  // owns a row's newest token writes the rotated k and v to the cache and into its staged page.
  int fused;
  int rope_mode;
  const void* rope_cos;
  const void* rope_sin;
  const __nv_bfloat16* qk_bias;
  __nv_bfloat16* kv;
  int64_t k_col, v_col;
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

// Element d of head vector x with the bias added in bf16 when present.
__device__ __forceinline__ float biased(const __nv_bfloat16* x, const __nv_bfloat16* b, int d) {
  const float v = bf16_to_f(x[d]);
  return b ? round_bf16(v + bf16_to_f(b[d])) : v;
}

// Rotation pair j of head vector x (bias b or null) at position pos: its element indices and
// rotated values, rounded to bf16 where the reference's ops round. Mode 1: Ouro split-half
// rotate_half with bf16 tables [pos][D]; mode 2: Huginn interleaved pairs in fp32 with fp32
// tables [pos][D/2] (modeling_huginn.py:178-196), each product and the sum rounded separately;
// mode 0: no rotation.
__device__ __forceinline__ void rope_pair(int mode, const void* rcos, const void* rsin, int pos, int D, int j,
                                          const __nv_bfloat16* x, const __nv_bfloat16* b, int& d0, int& d1,
                                          float& y0, float& y1) {
  if (mode == 1) {
    const int half = D / 2;
    d0 = j;
    d1 = j + half;
    const __nv_bfloat16* cr = static_cast<const __nv_bfloat16*>(rcos) + (int64_t)pos * D;
    const __nv_bfloat16* sr = static_cast<const __nv_bfloat16*>(rsin) + (int64_t)pos * D;
    const float x0 = biased(x, b, d0), x1 = biased(x, b, d1);
    y0 = rope_half(x0, x1, true, bf16_to_f(cr[d0]), bf16_to_f(sr[d0]));
    y1 = rope_half(x1, x0, false, bf16_to_f(cr[d1]), bf16_to_f(sr[d1]));
  } else if (mode == 2) {
    d0 = 2 * j;
    d1 = 2 * j + 1;
    const float c = static_cast<const float*>(rcos)[(int64_t)pos * (D / 2) + j];
    const float s = static_cast<const float*>(rsin)[(int64_t)pos * (D / 2) + j];
    const float x0 = biased(x, b, d0), x1 = biased(x, b, d1);
    y0 = round_bf16(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)));
    y1 = round_bf16(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s)));
  } else {
    d0 = 2 * j;
    d1 = 2 * j + 1;
    y0 = biased(x, b, d0);
    y1 = biased(x, b, d1);
  }
}

// The raw 16-byte operands of one 8-element RoPE chunk: the chunk, its bias, the split-half
// partner chunk and its bias (mode 1), and the cos/sin entries (8 bf16 for mode 1, 4 fp32 for
// mode 2). Loading and rotating are separate so the loads can be issued well before use.
struct RopeRaw {
  uint4 x, xb, px, pb, c, s;
};

__device__ __forceinline__ uint4 ld16(const void* ptr) { return *reinterpret_cast<const uint4*>(ptr); }

// Loads for dims [x0, x0 + 8) of head vector x (x0 a multiple of 8, so a chunk never straddles
// the split-half boundary or an interleaved pair; x, b and the tables 16-byte aligned).
__device__ __forceinline__ void rope_load(int mode, const void* rcos, const void* rsin, int pos, int D,
                                          const __nv_bfloat16* x, const __nv_bfloat16* b, int x0, RopeRaw& r) {
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  r.x = ld16(x + x0);
  r.xb = b ? ld16(b + x0) : z;
  r.px = r.pb = r.c = r.s = z;
  if (mode == 1) {
    const int px = x0 < D / 2 ? x0 + D / 2 : x0 - D / 2;
    r.px = ld16(x + px);
    r.pb = b ? ld16(b + px) : z;
    r.c = ld16(static_cast<const __nv_bfloat16*>(rcos) + (int64_t)pos * D + x0);
    r.s = ld16(static_cast<const __nv_bfloat16*>(rsin) + (int64_t)pos * D + x0);
  } else if (mode == 2) {
    r.c = ld16(static_cast<const float*>(rcos) + (int64_t)pos * (D / 2) + x0 / 2);
    r.s = ld16(static_cast<const float*>(rsin) + (int64_t)pos * (D / 2) + x0 / 2);
  }
}

__device__ __forceinline__ void unpack8(const uint4 w, float a[8]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    a[2 * k] = bf16lo(ws[k]);
    a[2 * k + 1] = bf16hi(ws[k]);
  }
}

__device__ __forceinline__ void add_bias8(float a[8], const uint4 b) {
  float t[8];
  unpack8(b, t);
#pragma unroll
  for (int e = 0; e < 8; ++e) a[e] = round_bf16(a[e] + t[e]);
}

// The rotated (and bias-added) chunk, exactly as rope_pair rotates each element. `low`: the
// chunk lies in the first half of the head vector.
__device__ __forceinline__ void rope_apply(int mode, bool has_bias, bool low, const RopeRaw& r, float y[8]) {
  float a[8];
  unpack8(r.x, a);
  if (has_bias) add_bias8(a, r.xb);
  if (mode == 1) {
    float pa[8], c[8], sn[8];
    unpack8(r.px, pa);
    if (has_bias) add_bias8(pa, r.pb);
    unpack8(r.c, c);
    unpack8(r.s, sn);
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = rope_half(a[e], pa[e], low, c[e], sn[e]);
  } else if (mode == 2) {
    const float cc[4] = {__uint_as_float(r.c.x), __uint_as_float(r.c.y), __uint_as_float(r.c.z), __uint_as_float(r.c.w)};
    const float sc[4] = {__uint_as_float(r.s.x), __uint_as_float(r.s.y), __uint_as_float(r.s.z), __uint_as_float(r.s.w)};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      y[2 * i] = round_bf16(__fsub_rn(__fmul_rn(a[2 * i], cc[i]), __fmul_rn(a[2 * i + 1], sc[i])));
      y[2 * i + 1] = round_bf16(__fadd_rn(__fmul_rn(a[2 * i + 1], cc[i]), __fmul_rn(a[2 * i], sc[i])));
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = a[e];
  }
}

__device__ __forceinline__ void rope_chunk8(int mode, const void* rcos, const void* rsin, int pos, int D,
                                            const __nv_bfloat16* x, const __nv_bfloat16* b, int x0, float y[8]) {
  RopeRaw r;
  rope_load(mode, rcos, rsin, pos, D, x, b, x0, r);
  rope_apply(mode, b != nullptr, x0 < D / 2, r, y);
}

// Fused append, producer side. A unit holding row `item`'s last page also writes the row's
// rotated k and its v for head group hg to cache row (last page, pos % 16): the producer warp
// issues the loads when it starts the unit (append_load), streams the unit's pages, then rotates
// and stores (append_store), so the load latency overlaps the page stream. The producer runs
// NSTAGE pages ahead of the consumers, so this costs them nothing.
template <int D, int HG>
struct AppendRegs {
  static constexpr int kChunks = HG * D / 8;  // 8-element chunks of the head group's k (and v)
  static constexpr int kPer = (kChunks + 31) / 32;
  RopeRaw k[kPer];
  uint4 v[kPer];
  int blk_id;
};

template <int D, int HG>
__device__ __forceinline__ void append_load(const AttnParams& p, int item, int hg, int pos, int blk_id,
                                            AppendRegs<D, HG>& a) {
  using A = AppendRegs<D, HG>;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* row = p.qkv + (int64_t)item * p.qkv_stride;
  a.blk_id = blk_id;
#pragma unroll
  for (int i = 0; i < A::kPer; ++i) {
    const int q = lane + 32 * i;
    if (q < A::kChunks) {
      const int head = hg * HG + q * 8 / D, x0 = q * 8 % D;
      const __nv_bfloat16* kb = p.qk_bias ? p.qk_bias + (int64_t)(p.num_heads + head) * D : nullptr;
      rope_load(p.rope_mode, p.rope_cos, p.rope_sin, pos, D, row + p.k_col + (int64_t)head * D, kb, x0, a.k[i]);
      a.v[i] = ld16(row + p.v_col + (int64_t)head * D + x0);
    }
  }
}

template <int D, int HG>
__device__ __forceinline__ void append_store(const AttnParams& p, int hg, int pos, const AppendRegs<D, HG>& a) {
  using A = AppendRegs<D, HG>;
  const int lane = threadIdx.x & 31;
  const int64_t crow = (int64_t)a.blk_id * kBlock + pos % kBlock;
  if (a.blk_id < 0 || crow >= p.kv_rows) {
    if (lane == 0) set_error(p.status, CDB_ERR_INDEX);
    return;
  }
  const int64_t hstride = (int64_t)p.num_heads * D;
  __nv_bfloat16* kd = p.kv + ((int64_t)(2 * p.cache_layer) * p.kv_rows + crow) * hstride + (int64_t)hg * HG * D;
  __nv_bfloat16* vd = kd + p.kv_rows * hstride;  // the V slice (cache index 2 * layer + 1), same row
#pragma unroll
  for (int i = 0; i < A::kPer; ++i) {
    const int q = lane + 32 * i;
    if (q < A::kChunks) {
      const int off = q * 8, x0 = off % D;  // head-group-relative offset; dim within the head
      float y[8];
      rope_apply(p.rope_mode, p.qk_bias != nullptr, x0 < D / 2, a.k[i], y);
      *reinterpret_cast<uint4*>(kd + off) = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                                                       pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
      *reinterpret_cast<uint4*>(vd + off) = a.v[i];
    }
  }
}

template <int D, int HG>
__global__ void __launch_bounds__(AttnCfg<D, HG>::THREADS) decode_attn_kernel(const __grid_constant__ CUtensorMap map,
                                                                              AttnParams p) {
  using C = AttnCfg<D, HG>;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NSTAGE * C::STAGE_BYTES);
  uint64_t* empty = full + C::NSTAGE;
  uint64_t* spec = empty + C::NSTAGE;  // completion of the speculative first pages
  float* merge = reinterpret_cast<float*>(spec + C::NSTAGE);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::CONSUMERS);
      mbar_init(&spec[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == C::CONSUMERS && lane == 0) prefetch_tensormap(&map);
  __syncthreads();
  pdl_trigger();
  // Speculative first pages (fused append only). The cached pages of positions below each row's
  // new token do not depend on the previous kernel, so before griddepcontrol.wait the producer
  // reads the plan, the block table and the first pages' block ids - as written by kernels that
  // may be still in flight, so possibly stale - and starts loading up to NSTAGE pages into the
  // ring, completing on `spec` instead of `full`. After the wait the producer walks the real
  // plan; a page whose (head group, block id) matches the speculated one is handed to the
  // consumers by a plain arrival on `full` once it has landed, any other page is loaded again
  // (after the speculative copy into its stage has landed). The new token's own position is never
  // read from a staged page in the fused mode, so a page loaded before its append is correct.
  int spec_n = 0, spec_hg = -1;
  int spec_ids[C::NSTAGE];
#pragma unroll
  for (int i = 0; i < C::NSTAGE; ++i) spec_ids[i] = -1;
  if (p.fused && warp == C::CONSUMERS && lane == 0) {
    const int nch = p.hdr[1];
    if ((int)blockIdx.x < nch && nch <= kMaxPlanChunks) {
      int u0, u1;
      chunk_units(p.hdr, blockIdx.x, u0, u1);
      if (u0 >= 0 && u0 < u1) {
        const Unit unit = decode_unit(p.units[u0]);
        const int slot = unit.row >= 0 && unit.row < p.num_items ? p.item_slot[unit.row] : -1;
        if (slot >= 0 && unit.b0 >= 0 && unit.b0 < unit.b1 && unit.b1 <= p.bt_stride) {
          const int32_t* bt = p.block_table + (int64_t)slot * p.bt_stride;
          spec_n = min(C::NSTAGE, unit.b1 - unit.b0);
          spec_hg = unit.hg;
          for (int i = 0; i < spec_n; ++i) {
            int id = bt[unit.b0 + i];
            if (id < 0 || (int64_t)(id + 1) * kBlock > p.kv_rows) id = 0;
            spec_ids[i] = id;
            mbar_arrive_expect_tx(&spec[i], C::STAGE_BYTES);
            uint8_t* dst = smem + i * C::STAGE_BYTES;
            tma_load_4d(dst, &map, &spec[i], 0, spec_hg * HG, id * kBlock, 2 * p.cache_layer);
            tma_load_4d(dst + C::TILE_BYTES, &map, &spec[i], 0, spec_hg * HG, id * kBlock, 2 * p.cache_layer + 1);
          }
        }
      }
    }
  }
  pdl_wait();

  const int n_chunks = p.hdr[1];

  if (warp == C::CONSUMERS) {
    // ------------------------------------------------------------- producer warp
    if (lane == 0) prefetch_tensormap(&map);
    int stage = 0;
    uint32_t phase = 0;
    bool alive = true;
    int issued = 0;  // pages handed to the ring so far (lane 0)
    for (int c = blockIdx.x; c < n_chunks && alive; c += gridDim.x) {
    int u0, u1;
    chunk_units(p.hdr, c, u0, u1);
    for (int u = u0; u < u1 && alive; ++u) {
      const Unit unit = decode_unit(p.units[u]);
      const int b0 = unit.b0;
      const int b1 = unit.b1;
      const int32_t* bt = p.block_table + (int64_t)p.item_slot[unit.row] * p.bt_stride;
      AppendRegs<D, HG> app;
      int app_pos = -1;
      if (p.fused) {
        const int pos = p.item_pos[unit.row];
        if (b1 == pos / kBlock + 1) {
          app_pos = pos;
          append_load<D, HG>(p, unit.row, unit.hg, pos, bt[b1 - 1], app);
        }
      }
      for (int base = b0; base < b1 && alive; base += 32) {
        const int my = base + lane < b1 ? bt[base + lane] : 0;
        const int cnt = min(32, b1 - base);
        for (int i = 0; i < cnt; ++i) {
          int block_id = __shfl_sync(0xffffffffu, my, i);
          if (lane == 0) {
            // A block id outside the pool (a -1 hole in the table or a stale id) is recorded
            // and page 0 is staged in its place, so the ring keeps its order; the output of
            // that row is then not meaningful and the status word says so.
            if (block_id < 0 || (int64_t)(block_id + 1) * kBlock > p.kv_rows) {
              set_error(p.status, CDB_ERR_INDEX);
              block_id = 0;
            }
            if (issued < spec_n) {
              // one of the speculative pages' stages: let that copy land before the stage is used
              if (!mbar_wait(&spec[issued], 0, p.status)) alive = false;
            }
            if (!alive) {
            } else if (issued < spec_n && spec_ids[issued] == block_id && spec_hg == unit.hg) {
              mbar_arrive(&full[stage]);  // the speculative copy is this page
            } else if (mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
              mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
              uint8_t* dst = smem + stage * C::STAGE_BYTES;
              tma_load_4d(dst, &map, &full[stage], 0, unit.hg * HG, block_id * kBlock, 2 * p.cache_layer);
              tma_load_4d(dst + C::TILE_BYTES, &map, &full[stage], 0, unit.hg * HG, block_id * kBlock,
                          2 * p.cache_layer + 1);
            } else {
              alive = false;
            }
            ++issued;
          }
          alive = __shfl_sync(0xffffffffu, alive, 0);
          if (!alive) break;
          if (++stage == C::NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (app_pos >= 0 && alive) append_store<D, HG>(p, unit.hg, app_pos, app);
    }
    }
    // no speculative copy may still be in flight when the CTA exits (bounded waits)
    if (lane == 0)
      for (int i = issued; i < spec_n; ++i) mbar_wait(&spec[i], 0, p.status);
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

    // this lane's q slice, rotated, pre-scaled by softmax_scale*log2(e)
    const __nv_bfloat16* qrow = p.qkv + (int64_t)item * p.qkv_stride + (int64_t)head * D;
    float qf[C::DPL];
    if (p.fused) {
      const __nv_bfloat16* qb = p.qk_bias ? p.qk_bias + (int64_t)head * D : nullptr;
#pragma unroll
      for (int c = 0; c < C::NCH; ++c) {
        float y[8];
        rope_chunk8(p.rope_mode, p.rope_cos, p.rope_sin, pos, D, qrow, qb, (c * C::LPT + cq) * 8, y);
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[c * 8 + e] = y[e] * p.scale_log2;
      }
    } else {
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
    }

    // Fused append: the piece holding the row's last page stages that page before position pos
    // is written, so the warp whose token half holds pos takes that token from registers: its
    // score is q . k_new summed in the page loop's order (bit-identical to reading k_new from the
    // page) and its value pairs are v_new. The producer warp writes k_new and v_new to the cache
    // row (append_load / append_store); no unit of the launch reads that row from the cache.
    const int t_new = pos % kBlock;
    const bool owner = p.fused && b1 == pos / kBlock + 1 && sub == t_new / C::TPW;
    float kdot_new = 0.f;
    uint32_t vnew[C::PPL];
#pragma unroll
    for (int i = 0; i < C::PPL; ++i) vnew[i] = 0u;
    if (owner) {
      const __nv_bfloat16* krow_g = p.qkv + (int64_t)item * p.qkv_stride + p.k_col + (int64_t)head * D;
      const __nv_bfloat16* vrow_g = p.qkv + (int64_t)item * p.qkv_stride + p.v_col + (int64_t)head * D;
      const __nv_bfloat16* kb = p.qk_bias ? p.qk_bias + (int64_t)(p.num_heads + head) * D : nullptr;
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
      for (int c = 0; c < C::NCH; ++c) {
        const int x0 = (c * C::LPT + cq) * 8;
        float y[8];
        rope_chunk8(p.rope_mode, p.rope_cos, p.rope_sin, pos, D, krow_g, kb, x0, y);
        acc0 = fmaf(qf[c * 8 + 0], y[0], acc0);
        acc1 = fmaf(qf[c * 8 + 1], y[1], acc1);
        acc0 = fmaf(qf[c * 8 + 2], y[2], acc0);
        acc1 = fmaf(qf[c * 8 + 3], y[3], acc1);
        acc0 = fmaf(qf[c * 8 + 4], y[4], acc0);
        acc1 = fmaf(qf[c * 8 + 5], y[5], acc1);
        acc0 = fmaf(qf[c * 8 + 6], y[6], acc0);
        acc1 = fmaf(qf[c * 8 + 7], y[7], acc1);
      }
      kdot_new = acc0 + acc1;
#pragma unroll
      for (int i = 0; i < C::PPL; ++i) {
        const int j = lane + 32 * i;
        if (j < C::NPAIR) vnew[i] = *reinterpret_cast<const uint32_t*>(vrow_g + 2 * j);
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
        const bool last_own = owner && blk == b1 - 1;
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
          if (last_own && t == t_new) acc = kdot_new;
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
              const uint32_t w = (last_own && t == t_new) ? vnew[i] : vrow[(t * HG + hh) * C::NPAIR + j];
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
#pragma unroll 4
    for (int sp = 0; sp < nsplit; ++sp) mx = fmaxf(mx, __ldcg(p.part_ml + 2 * (base + sp)));
    float lsum = 0.f;
    float acc[2 * C::PPL];
#pragma unroll
    for (int i = 0; i < 2 * C::PPL; ++i) acc[i] = 0.f;
#pragma unroll 4
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
  for (int i = threadIdx.x; i < num_heads * half; i += blockDim.x) {
    const int h = i / half, j = i % half;
    const int64_t hb = (int64_t)h * D;
    int d0, d1;
    float y0, y1;
    if (rope_mode != 0 || qk_bias) {
      rope_pair(rope_mode, rope_cos, rope_sin, pos, D, j, q + hb, qk_bias ? qk_bias + hb : nullptr, d0, d1, y0, y1);
      q[hb + d0] = f_to_bf16(y0);
      q[hb + d1] = f_to_bf16(y1);
    }
    rope_pair(rope_mode, rope_cos, rope_sin, pos, D, j, k + hb, kb ? kb + hb : nullptr, d0, d1, y0, y1);
    kd[hb + d0] = f_to_bf16(y0);
    kd[hb + d1] = f_to_bf16(y1);
    vd[hb + d0] = v[hb + d0];
    vd[hb + d1] = v[hb + d1];
  }
}

// Vectorised rope + append: one CTA per row, one thread per 8-element chunk of the H*D q (and k, v)
// vector, 16-byte loads and stores. Every q chunk is read before any is rewritten in place (the
// split-half rotation reads a partner chunk another thread owns). Same arithmetic as
// rope_append_kernel (rope_load / rope_apply restate rope_pair per chunk).
// One CTA per row, one thread per 8-element chunk of the row's heads. Rows of up to 256 chunks
// (16 heads x 128) take the MAXT = 256 instantiation, bounded to 64 registers so four CTAs stay
// resident per SM (the unbounded build took 68 and fit three); the kernel is latency-bound, one
// row per CTA behind a chain of index loads. Wider rows (55 heads x 96) take MAXT = 1024, whose
// bound also keeps a 1024-thread launch within the SM's 65,536 registers.
template <int MAXT>
__global__ void __launch_bounds__(MAXT, (MAXT <= 256 ? 4 : 1))
    rope_append_vec_kernel(__nv_bfloat16* qkv, int64_t qkv_stride, int64_t k_col, int64_t v_col,
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
  const int c = threadIdx.x;
  const bool active = c < num_heads * D / 8;
  const int head = active ? c * 8 / D : 0, x0 = active ? c * 8 % D : 0;
  const int64_t hb = (int64_t)head * D;
  const bool rot_q = rope_mode != 0 || qk_bias != nullptr;
  RopeRaw rq, rk;
  uint4 vv = make_uint4(0u, 0u, 0u, 0u);
  if (active) {
    if (rot_q) rope_load(rope_mode, rope_cos, rope_sin, pos, D, q + hb, qk_bias ? qk_bias + hb : nullptr, x0, rq);
    rope_load(rope_mode, rope_cos, rope_sin, pos, D, k + hb, qk_bias ? qk_bias + hstride + hb : nullptr, x0, rk);
    vv = ld16(v + hb + x0);
  }
  __syncthreads();
  if (!active) return;
  float y[8];
  if (rot_q) {
    rope_apply(rope_mode, qk_bias != nullptr, x0 < D / 2, rq, y);
    *reinterpret_cast<uint4*>(q + hb + x0) = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                                                        pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
  }
  rope_apply(rope_mode, qk_bias != nullptr, x0 < D / 2, rk, y);
  *reinterpret_cast<uint4*>(kd + hb + x0) = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                                                       pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
  *reinterpret_cast<uint4*>(vd + hb + x0) = vv;
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
  const int chunks = num_heads * head_dim / 8;
  const bool aligned16 = ((reinterpret_cast<uintptr_t>(qk_bias) | reinterpret_cast<uintptr_t>(kv_base) |
                           reinterpret_cast<uintptr_t>(qkv)) & 15) == 0 &&
                         (rope_mode == 0 ||
                          ((reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin)) & 15) == 0) &&
                         (qkv_stride & 7) == 0 && (k_col & 7) == 0 && (v_col & 7) == 0;
  if (head_dim % 8 == 0 && chunks <= 1024 && aligned16) {
    const int threads = ((chunks + 31) / 32) * 32;
    auto* kern = threads <= 256 ? rope_append_vec_kernel<256> : rope_append_vec_kernel<1024>;
    return launch_pdl(kern, dim3(num_items), dim3(threads), 0, st, static_cast<__nv_bfloat16*>(qkv), qkv_stride, k_col,
                      v_col, static_cast<__nv_bfloat16*>(kv_base), kv_rows, cache_layer, block_table, bt_stride,
                      item_slot, item_pos, rope_mode, rope_cos, rope_sin, static_cast<const __nv_bfloat16*>(qk_bias),
                      num_heads, head_dim, status) == cudaSuccess
               ? CDB_OK
               : CDB_ERR_CUDA;
  }
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
  if (rope_mode < 0 || rope_mode > 2 || append < 0 || append > 2 ||
      (append && rope_mode != 0 && (rope_cos == nullptr || rope_sin == nullptr)))
    return CDB_ERR_INVALID_ARGUMENT;
  // the fused append reads tables and bias in 16-byte vectors
  if (append == 2 && ((reinterpret_cast<uintptr_t>(qk_bias) & 15) ||
                      (rope_mode != 0 && ((reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin)) & 15))))
    return CDB_ERR_INVALID_ARGUMENT;
  (void)scratch_items;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (append == 1) {
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
  p.num_items = num_items;
  p.scale_log2 = scale * kLog2e;
  p.status = status;
  p.fused = append == 2;
  p.rope_mode = rope_mode;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  p.qk_bias = static_cast<const __nv_bfloat16*>(qk_bias);
  p.kv = static_cast<__nv_bfloat16*>(kv_base);
  p.k_col = k_col;
  p.v_col = v_col;
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
  if (rope_mode < 0 || rope_mode > 2 || append < 0 || append > 2 ||
      (append && rope_mode != 0 && (rope_cos == nullptr || rope_sin == nullptr)))
    return CDB_ERR_INVALID_ARGUMENT;
  // the fused append reads tables and bias in 16-byte vectors
  if (append == 2 && ((reinterpret_cast<uintptr_t>(qk_bias) & 15) ||
                      (rope_mode != 0 && ((reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin)) & 15))))
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
  if (append == 1) {
    rc = launch_rope_append(qkv, qkv_stride, k_col, v_col, kv_base, kv_rows, cache_layer, block_table,
                            block_table_stride, item_slot, item_pos, rope_mode, rope_cos, rope_sin, qk_bias,
                            num_items, num_heads, head_dim, status, st);
    if (rc != CDB_OK) return rc;
  }
  // One plan chunk per attention CTA; the plan holds at most CDB_ATTN_PLAN_MAX_CHUNKS chunks, so
  // the grid is clamped to that too (a wider grid would only add CTAs without work).
  if (num_ctas <= 0) num_ctas = 2 * 148;
  num_ctas = num_ctas < kMaxPlanChunks ? num_ctas : kMaxPlanChunks;
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
  p.num_items = num_items;
  p.scale_log2 = scale * kLog2e;
  p.status = status;
  p.fused = append == 2;
  p.rope_mode = rope_mode;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  p.qk_bias = static_cast<const __nv_bfloat16*>(qk_bias);
  p.kv = static_cast<__nv_bfloat16*>(kv_base);
  p.k_col = k_col;
  p.v_col = v_col;
  if (head_dim == 128) return launch_attn<128, 4>(map, p, num_ctas, st);
  if (head_dim == 64) return launch_attn<64, 4>(map, p, num_ctas, st);
  if (head_dim == 96) return launch_attn<96, 5>(map, p, num_ctas, st);
  return CDB_ERR_UNSUPPORTED;
}
