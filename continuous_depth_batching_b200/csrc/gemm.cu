// bf16 tensor-core GEMM for sm_100a on tcgen05/TMEM: C[M,N] = X[M,K] * W[N,K]^T.
//
// Orientation. Decode-shaped problems have few token rows (M <= 256) and wide weights (N up to
// 65536), so the weight is the MMA "A" operand (128 weight rows per tile, UMMA M = 128) and the
// token rows are the MMA "B" operand (UMMA N = BN, M rounded up to 16, at most 256); the fp32
// accumulator lives in tensor memory as [128 lanes = weight rows] x [BN columns = token rows].
// Prefill-shaped problems tile the tokens by 256.
//
// Work split (stream-K). The launch has G = min(#SMs, iterations) CTAs, one per SM (two per SM
// for token tiles narrower than 128, each with a smaller ring). The iteration space - every
// (output tile, 64-wide k block) pair, tiles in token-major order - is cut into G equal contiguous
// ranges, so every SM streams the same number of bytes whatever the tile count. A CTA's range
// covers the tail of one tile, whole tiles and the head of another; a tile covered by one CTA is
// stored directly. A tile split over CTAs belongs to the CTA holding its first k block (for that
// CTA it is the range's last segment); every other piece is the first segment of a later range.
// Those pieces write their fp32 partial to the caller's workspace and bump the tile's counter;
// the owner waits for the counter (bounded), bulk-copies the pieces into its now idle rings and
// adds them to its own accumulator in CTA order (so the result does not depend on timing), runs
// the epilogue and resets the counter. Owners wait only on later CTAs' first segments, which wait
// on nothing, so the waits cannot form a cycle; all G CTAs are co-resident by construction.
//
// Tiles: above 256 tokens the plain and argmax epilogues use 256 weight rows x 256 tokens (two
// 128-row accumulators sharing every activation tile); otherwise 128 weight rows x BN tokens with
// two TMEM buffers, so one tile's epilogue overlaps the next tile's main loop.
//
// Warp roles (224 threads):
//   warp 0      weight producer: 2-D TMA tile loads W[128 x 64] (128-byte swizzle) into an SW-deep
//               ring. Weights do not depend on the previous kernel, so this warp never waits for
//               it: with programmatic dependent launch the weight stream starts while the
//               predecessor is still finishing.
//   warp 1      activation producer: waits for the predecessor (griddepcontrol.wait), then loads
//               X[BN x 64] tiles into an SX-deep ring.
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each warp its 32-lane quarter) and emit it
//               through a shared-memory staging tile as 16-byte stores, or publish / combine
//               split pieces.
//   warp 6      allocates TMEM and issues tcgen05.mma from one thread.
// Every role branch ends converged (__syncwarp) before the final block barrier, which guards the
// TMEM free.
// Epilogues: 0 stores bf16(C); 1 (SwiGLU) reads weight rows as gate/up pairs and stores
// bf16(bf16(silu(bf16(g))) * bf16(u)); 2 (LM head + greedy argmax) stores no logits: each CTA
// keeps its best 64-bit (logit, index) key per token in shared memory, folds it into the global
// keys with one atomicMax per token and token tile, and the last CTA writes the token ids.
// Every wait is bounded; a wait that runs out records CDB_ERR_DEVICE_TIMEOUT and the CTA winds
// down.
//
// Split mode (gemm_cluster.cuh). When a problem has fewer output tiles than SMs (every
// decode-shaped projection), stream-K would cut each tile into many pieces and leave one CTA to
// read them all back; there the K range of each tile is split over a thread-block cluster whose
// ranks reduce the partial tile through distributed shared memory instead.
//
// Pair mode (gemm_pair.cuh). Above 256 tokens, with at least two 256 x 256 tiles per pair of SMs,
// the plain and SwiGLU epilogues run on 2-CTA clusters issuing tcgen05.mma.cta_group::2: each CTA
// holds half of a 256 x 256 accumulator, which leaves TMEM room for two buffers, and the work is
// stream-K over the pairs. The one-SM stream-K kernel below serves the LM head and the problems
// pair mode does not take.
#include <cooperative_groups.h>
#include <cuda.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "cdb_common.cuh"

namespace cdb {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle atom of bf16
constexpr int W_BYTES = BM * BK * 2;
constexpr int THREADS = 7 * 32;
constexpr int kWarpW = 0, kWarpX = 1, kWarpMma = 6;
constexpr int kEpiThreads = 128;
constexpr int kSmemBudget = 200 * 1024;
constexpr int kNarrowRing = 88 * 1024;  // ring bytes of a narrow-token-tile CTA (two CTAs per SM)
constexpr int kStgPitch = (BM + 8) * 2;  // bytes per staged token row (16-byte aligned, bank-skewed)
constexpr int kStgBytes = 32 * kStgPitch;

constexpr int cmin(int a, int b) { return a < b ? a : b; }
constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int pow2_at_least(int v) { return v <= 32 ? 32 : v <= 64 ? 64 : v <= 128 ? 128 : 256; }

// WM = weight tiles per CTA tile: 1 (128 weight rows; two TMEM accumulator buffers, so the
// epilogue of one tile overlaps the main loop of the next) or 2 (256 weight rows x 256 tokens for
// prefill: two accumulators sharing every activation tile, which cuts the shared-memory fill per
// FLOP by a third; one buffer, the epilogue runs between tiles).
template <int BN, int WM = 1>
struct Cfg {
  static constexpr int X_BYTES = BN * BK * 2;
  static constexpr int W_STAGE = WM * W_BYTES;
  // Rings: wide token tiles split the budget evenly (prefill is MMA-bound and needs both operands
  // deep). Narrow ones (decode widths: the LM head, wide SwiGLU projections) run two CTAs per SM,
  // each with a 3-deep activation ring (X is L2-resident) and ~88 KB of weight ring: two CTAs
  // streaming per SM pulled the Huginn-0125 LM head (65536 x 5280) at 5.1 TB/s against 4.4 TB/s
  // for one CTA with a 12-deep ring.
  static constexpr int SX = BN >= 128 ? kSmemBudget / (W_STAGE + X_BYTES) : 3;
  static constexpr int SW = BN >= 128 ? SX : cmin(12, (kNarrowRing - SX * X_BYTES) / W_STAGE);
  static constexpr int ACC_STRIDE = pow2_at_least(BN);  // TMEM columns of one 128-row accumulator
  static constexpr int NBUF = WM == 1 ? 2 : 1;          // accumulator buffers
  static constexpr int ACC_SPAN = WM * ACC_STRIDE;      // TMEM columns of one buffer
  static constexpr uint32_t TMEM_COLS = NBUF * ACC_SPAN;
  static constexpr int TM = WM * BM;  // weight rows per CTA tile
  static constexpr int CHUNKS = (BN + 31) / 32;
  static constexpr int OFF_X = SW * W_STAGE;
  static constexpr int OFF_BAR = OFF_X + SX * X_BYTES;
  static constexpr int NBAR = 2 * SW + 2 * SX + 7;  // rings, 2 accumulator x 2, drain, 2 fixup
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_KEYS = (OFF_MISC + 64 + 7) / 8 * 8;  // argmax: [4 warps][32] keys, then [BN] best
  static constexpr int OFF_STG = (OFF_KEYS + (4 * 32 + BN) * 8 + 15) / 16 * 16;  // 2 staging tiles
  static constexpr int SMEM = OFF_STG + 2 * kStgBytes + 1024;                      // + alignment slack
  // kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, M=128, N=BN.
  static constexpr uint32_t IDESC =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
  static_assert(WM == 1 || BN == 256, "two weight tiles per CTA tile only for 256-token tiles");
  static_assert(TMEM_COLS <= 512, "TMEM");
  static_assert(SX >= 2 && SW >= 2, "rings");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(BN >= 128 || 2 * (SMEM + 1024) <= 228 * 1024, "narrow token tiles: two CTAs per SM");
  static_assert(X_BYTES % 1024 == 0, "swizzled X stages stay 1024-byte aligned");
};

struct Params {
  __nv_bfloat16* c;
  int64_t ldc;
  int M, N, K;
  int tiles_w, tiles_tok, kb;  // weight tiles, token tiles, k blocks per tile
  long long iters;             // tiles * kb
  float* ws;                   // split partials: [2 * G][WM * BM * BN] fp32
  int32_t* ctr;                // per-tile arrival counters (zero between calls)
  int pair_store;              // EPI 0: c 4-byte aligned, ldc and N even (EPI 1: act 4-byte aligned, ldc even)
  int vec_store;               // split mode EPI 0: c 8-byte aligned, ldc % 4 == 0
  int vec16;                   // stream-K EPI 0/1: c 16-byte aligned, ldc % 8 == 0
  int32_t* status;
  // EPI 2 (LM head + argmax)
  unsigned long long* keys;
  int32_t* done;
  int64_t* out_ids;
  const int32_t* out_rows;
  const int32_t* token_rows;
  int32_t* token_table;
};

// Orderable 64-bit key of (bf16 logit v, vocab index n): larger v wins, then the smaller index
// (torch.argmax returns the first maximum). 0 is below every real key.
__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)n);
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of 128 B,
// 8-row groups 1024 B apart (SBO), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  const uint32_t mask0 = 0, mask1 = 0, mask2 = 0, mask3 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2), "r"(mask3)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"r"(kEpiThreads) : "memory"); }

__device__ __forceinline__ float4 ld_cg_f4(const float4* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Bounded mbarrier wait that also gives up once another role of the CTA has given up.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, int32_t* status, volatile int* abort) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort) return false;
  }
  set_error(status, CDB_ERR_DEVICE_TIMEOUT);
  *abort = 1;
  return false;
}

// Iteration range start of CTA g, and the CTA whose range holds iteration x.
__device__ __forceinline__ long long range_start(long long iters, int G, int g) { return iters * g / G; }
__device__ __forceinline__ int cta_of(long long iters, int G, long long x) { return (int)(((x + 1) * G - 1) / iters); }

// Workspace slot of CTA g's piece of tile t: its first piece (the range starts inside tile t) or
// its last one. Slot layout: float4 index (chunk * 8 + j / 4) * BM + row holds tokens j..j+3 of
// the chunk for one weight row, so a warp moves 512 contiguous bytes per access.
__device__ __forceinline__ int piece_slot(long long iters, int G, int g, long long tile_begin) {
  return range_start(iters, G, g) >= tile_begin ? 2 * g : 2 * g + 1;
}

// Bulk copy global -> shared (async proxy), completing on an mbarrier's transaction count.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ int ld_acquire(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Emit one 32-token chunk of a finished tile. v[j] = accumulator of weight row n0 + row (this
// thread's TMEM lane) and token m0 + j (in-tile column col0 + j, valid below BN).
//   EPI 0: bf16 values go through a [32 token][128 row] staging tile in shared memory and leave as
//          16-byte stores, 256 contiguous bytes per token row.
//   EPI 1: weight rows (2i, 2i+1) = (gate_i, up_i) sit on lanes (2l, 2l+1); the pair stages
//          act[token][i] (64 columns per 128 rows), stored the same way.
//   EPI 2: no logits: the best (logit, index) key of every token over the 128 rows is folded into
//          the CTA's per-token best (s_best), flushed to the global keys once per token tile.
// One named barrier per chunk; the staging tile alternates between two buffers, so a buffer is
// rewritten only after every thread has passed the next chunk's barrier.

template <int BN, int EPI>
__device__ __forceinline__ void emit_chunk(const Params& p, const float (&v)[32], int n0, int row, int m0, int col0,
                                           int lane, int q, int et, uint8_t* stg, unsigned long long* s_keys,
                                           unsigned long long* s_best) {
  if constexpr (EPI == 0 || EPI == 1) {
    __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(stg);
    constexpr int kRowElems = kStgPitch / 2;
    if constexpr (EPI == 0) {
#pragma unroll
      for (int j = 0; j < 32; ++j) st[j * kRowElems + row] = f_to_bf16(v[j]);
    } else {
      // lanes 2l and 2l+1 split the chunk's tokens: the even lane takes the even tokens and the
      // odd lane the odd ones, one shuffle per token pair
      const int odd = lane & 1;
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float x = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
        const float g = round_bf16(odd ? x : v[j]), u = round_bf16(odd ? v[j + 1] : x);
        const float s = round_bf16(g / (1.f + expf(-g)));
        st[(j + odd) * kRowElems + row / 2] = f_to_bf16(s * u);
      }
    }
    epi_bar();
    // output columns of this chunk: [c0, c0 + cols) of a row-major [M, ncols] matrix
    constexpr int cols = EPI == 0 ? BM : BM / 2;
    constexpr int vecs = cols / 8;  // 16-byte vectors per token row
    const int c0 = EPI == 0 ? n0 : n0 / 2;
    const int ncols = EPI == 0 ? p.N : p.N / 2;
#pragma unroll
    for (int k = 0; k < 32 * vecs / kEpiThreads; ++k) {
      const int idx = et + k * kEpiThreads;
      const int tok = idx / vecs, vc = idx % vecs;
      const int m = m0 + tok, n = c0 + vc * 8;
      if (col0 + tok >= BN || m >= p.M || n >= ncols) continue;
      const uint4 val = *reinterpret_cast<const uint4*>(stg + tok * kStgPitch + vc * 16);
      __nv_bfloat16* dst = p.c + (int64_t)m * p.ldc + n;
      if (p.vec16 && n + 8 <= ncols) {
        *reinterpret_cast<uint4*>(dst) = val;
      } else {
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&val);
        for (int i = 0; i < 8 && n + i < ncols; ++i) dst[i] = e[i];
      }
    }
  } else {
    // Transpose-reduce: after 5 butterfly stages lane l holds the best key of chunk token l over
    // the warp's 32 rows; the 4 epilogue warps then meet in shared memory.
    (void)stg;
    (void)et;
    const int n = n0 + row;
    unsigned long long k[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const bool ok = col0 + j < BN && m0 + j < p.M && n < p.N;
      k[j] = ok ? argmax_key(round_bf16(v[j]), n) : 0ull;
    }
#pragma unroll
    for (int h = 16; h >= 1; h >>= 1) {
      const bool upper = (lane & h) != 0;
#pragma unroll
      for (int i = 0; i < h; ++i) {
        const unsigned long long keep = upper ? k[i + h] : k[i];
        const unsigned long long send = upper ? k[i] : k[i + h];
        const unsigned long long got = __shfl_xor_sync(0xffffffffu, send, h);
        k[i] = keep > got ? keep : got;
      }
    }
    s_keys[q * 32 + lane] = k[0];
    epi_bar();
    if (q == 0 && col0 + lane < BN) {
      unsigned long long best = s_best[col0 + lane];
#pragma unroll
      for (int w = 0; w < 4; ++w) best = s_keys[w * 32 + lane] > best ? s_keys[w * 32 + lane] : best;
      s_best[col0 + lane] = best;
    }
    epi_bar();
  }
}

// EPI 2: fold the CTA's per-token best keys of token tile starting at mbase into the global keys
// (one atomicMax per token and CTA) and clear them. Called by all epilogue threads.
template <int BN>
__device__ __forceinline__ void flush_keys(const Params& p, unsigned long long* s_best, int mbase, int et) {
  epi_bar();
  for (int j = et; j < BN; j += kEpiThreads) {
    const unsigned long long b = s_best[j];
    if (b != 0ull && mbase + j < p.M) atomicMax(p.keys + mbase + j, b);
    s_best[j] = 0ull;
  }
  epi_bar();
}

template <int BN, int EPI, int WM>
__global__ void __launch_bounds__(THREADS, (BN < 128 ? 2 : 1))
    gemm_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, Params p) {
  using C = Cfg<BN, WM>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wring = smem;
  uint8_t* xring = smem + C::OFF_X;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* wempty = wfull + C::SW;
  uint64_t* xfull = wempty + C::SW;
  uint64_t* xempty = xfull + C::SX;
  uint64_t* afull = xempty + C::SX;
  uint64_t* aempty = afull + 2;
  uint64_t* mdrain = aempty + 2;  // the MMA issuer's last commit: every MMA done before TMEM is freed
  uint64_t* fbar = mdrain + 1;    // [2] owner fixup: bulk copies of the other pieces
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);
  volatile int* s_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 16);
  unsigned long long* s_keys = reinterpret_cast<unsigned long long*>(smem + C::OFF_KEYS);
  unsigned long long* s_best = s_keys + 4 * 32;  // EPI 2: the CTA's best key per token of a token tile
  uint8_t* stg = smem + C::OFF_STG;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int g = blockIdx.x;
  const long long it0 = range_start(p.iters, G, g);
  const long long it1 = range_start(p.iters, G, g + 1);
  const int kb = p.kb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::SW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int s = 0; s < C::SX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int b = 0; b < C::NBUF; ++b) {
      mbar_init(&afull[b], 1);
      mbar_init(&aempty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(mdrain, 1);
    mbar_init(&fbar[0], 1);
    mbar_init(&fbar[1], 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == kWarpW) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0) {
      prefetch_tensormap(&map_w);
      long long i = 0;
      for (long long it = it0; it < it1; ++it, ++i) {
        const int t = (int)(it / kb), k = (int)(it % kb);
        const int wt = t % p.tiles_w;
        const int s = (int)(i % C::SW);
        if (!wait_or_abort(&wempty[s], (uint32_t)(((i / C::SW) & 1) ^ 1), p.status, s_abort)) break;
        mbar_arrive_expect_tx(&wfull[s], C::W_STAGE);
#pragma unroll
        for (int w = 0; w < WM; ++w)
          tma_load_2d(wring + s * C::W_STAGE + w * W_BYTES, &map_w, &wfull[s], k * BK, wt * C::TM + w * BM);
      }
      // no copy may still be in flight when the CTA exits (bounded waits that ignore an abort)
      for (long long j = (i > C::SW ? i - C::SW : 0); j < i; ++j)
        mbar_wait(&wfull[j % C::SW], (uint32_t)((j / C::SW) & 1), p.status);
    }
    __syncwarp();  // the warp reaches the final block barrier converged
  } else if (warp == kWarpX) {
    // ------------------------------------------------------------ activation producer
    if (lane == 0) {
      prefetch_tensormap(&map_x);
      pdl_wait();
      long long i = 0;
      for (long long it = it0; it < it1; ++it, ++i) {
        const int t = (int)(it / kb), k = (int)(it % kb);
        const int tt = t / p.tiles_w;
        const int s = (int)(i % C::SX);
        if (!wait_or_abort(&xempty[s], (uint32_t)(((i / C::SX) & 1) ^ 1), p.status, s_abort)) break;
        mbar_arrive_expect_tx(&xfull[s], C::X_BYTES);
        tma_load_2d(xring + s * C::X_BYTES, &map_x, &xfull[s], k * BK, tt * BN);
      }
      for (long long j = (i > C::SX ? i - C::SX : 0); j < i; ++j)
        mbar_wait(&xfull[j % C::SX], (uint32_t)((j / C::SX) & 1), p.status);
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      long long i = 0;
      int seg = 0;
      bool ok = true;
      for (long long it = it0; it < it1 && ok; ++seg) {
        const long long t = it / kb;
        const long long seg_end = (t + 1) * kb < it1 ? (t + 1) * kb : it1;
        const int buf = seg % C::NBUF;
        if (!wait_or_abort(&aempty[buf], (uint32_t)(((seg / C::NBUF) & 1) ^ 1), p.status, s_abort)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * C::ACC_SPAN);
        for (bool first = true; it < seg_end; ++it, ++i, first = false) {
          const int ws = (int)(i % C::SW), xs = (int)(i % C::SX);
          if (!wait_or_abort(&wfull[ws], (uint32_t)((i / C::SW) & 1), p.status, s_abort) ||
              !wait_or_abort(&xfull[xs], (uint32_t)((i / C::SX) & 1), p.status, s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(wring + ws * C::W_STAGE);
          const uint32_t b = smem_u32(xring + xs * C::X_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
#pragma unroll
            for (int w = 0; w < WM; ++w)
              umma_bf16(d + (uint32_t)(w * C::ACC_STRIDE), sw128_desc(a + w * W_BYTES + kk * 32), sw128_desc(b + kk * 32),
                        C::IDESC, (!first || kk > 0) ? 1u : 0u);
          umma_commit(&wempty[ws]);
          umma_commit(&xempty[xs]);
        }
        if (ok) umma_commit(&afull[buf]);
      }
      // On every path (an abandoned wait included) no MMA may still run when TMEM is freed.
      umma_commit(mdrain);
      mbar_wait(mdrain, 0, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int et = threadIdx.x - 64;
    const int row = q * 32 + lane;
    pdl_wait();  // outputs, workspace and counters may still be in use by the predecessor
    if constexpr (EPI == 2) {
      for (int j = et; j < BN; j += kEpiThreads) s_best[j] = 0ull;
    }
    int seg = 0, emitted = 0, best_tt = -1;
    for (long long it = it0; it < it1; ++seg) {
      const long long t = it / kb;
      const long long tile_begin = t * kb;
      const long long seg_end = (t + 1) * kb < it1 ? (t + 1) * kb : it1;
      const bool full = it == tile_begin && seg_end == tile_begin + kb;
      it = seg_end;
      const int buf = seg % C::NBUF;
      if (et == 0) *s_flag = wait_or_abort(&afull[buf], (uint32_t)((seg / C::NBUF) & 1), p.status, s_abort) ? 1 : 0;
      epi_bar();
      if (!*s_flag) break;
      epi_bar();  // everyone has read the flag before it is reused
      tc_fence_after();
      const int wt = (int)(t % p.tiles_w), tt = (int)(t / p.tiles_w);
      const int mbase = tt * BN;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * C::ACC_SPAN);
      if constexpr (EPI == 2) {
        if (tt != best_tt) {
          if (best_tt >= 0) flush_keys<BN>(p, s_best, best_tt * BN, et);
          best_tt = tt;
        }
      }
      if (full) {
        // Whole tile in this CTA: emit chunk by chunk, then release the buffer (the MMA warp
        // meanwhile fills the other one, when there are two).
#pragma unroll 1
        for (int hc = 0; hc < WM * C::CHUNKS; ++hc, ++emitted) {
          const int w = hc / C::CHUNKS, c = hc % C::CHUNKS;
          float v[32];
          tmem_ld32(taddr + w * C::ACC_STRIDE + c * 32, v);
          emit_chunk<BN, EPI>(p, v, wt * C::TM + w * BM, row, mbase + c * 32, c * 32, lane, q, et,
                              stg + (emitted & 1) * kStgBytes, s_keys, s_best);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&aempty[buf]);
        continue;
      }
      // Split tile. Its owner is the CTA holding the tile's first k block: the tile is the last
      // segment of the owner's range, while every other piece is the first segment of a later
      // range, so the other pieces are (nearly) done when the owner gets here.
      const int ga = cta_of(p.iters, G, tile_begin);
      const int gb = cta_of(p.iters, G, tile_begin + kb - 1);
      // piece layout in a workspace slot: float4 ((w * BN / 4) + chunk * 8 + j / 4) * BM + row
      if (g != ga) {
        float4* mine = reinterpret_cast<float4*>(p.ws + (size_t)piece_slot(p.iters, G, g, tile_begin) * (C::TM * BN));
#pragma unroll 1
        for (int hc = 0; hc < WM * C::CHUNKS; ++hc) {
          const int w = hc / C::CHUNKS, c = hc % C::CHUNKS;
          float v[32];
          tmem_ld32(taddr + w * C::ACC_STRIDE + c * 32, v);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            if (c * 32 + j4 * 4 < BN)
              mine[(w * (BN / 4) + c * 8 + j4) * BM + row] =
                  make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&aempty[buf]);
        __threadfence();
        epi_bar();
        if (et == 0) atomicAdd(p.ctr + t, 1);
        continue;
      }
      // Owner: wait until the other gb - ga pieces are published, then add them in CTA order to
      // this CTA's own accumulator (own + piece(ga+1) + ... + piece(gb): the same order in every
      // run). The W and X rings are idle now (this is the range's last segment and every MMA has
      // completed), so the pieces come into shared memory by bulk copies, double-buffered in
      // batches of chunks.
      const int others = gb - ga;
      if (et == 0) {
        bool ok = false;
        for (uint32_t i = 0; i < (kSpinLimit >> 4); ++i) {
          if (ld_acquire(p.ctr + t) >= others) {
            ok = true;
            break;
          }
          if (*s_abort) break;
          __nanosleep(64);
        }
        if (ok) {
          p.ctr[t] = 0;  // every piece has arrived: ready for the next call
          asm volatile("fence.proxy.async.global;" ::: "memory");
        } else {
          set_error(p.status, CDB_ERR_DEVICE_TIMEOUT);
          *s_abort = 1;
        }
        *s_flag = ok ? 1 : 0;
      }
      epi_bar();
      if (!*s_flag) break;
      epi_bar();
      constexpr int kChunkBytes = BM * 32 * 4;   // one 32-column chunk of a 128-row piece
      constexpr int kHalf = C::OFF_BAR / 2;      // half of the ring bytes
      constexpr int kTotalChunks = WM * C::CHUNKS;
      const int batch = kHalf / (others * kChunkBytes);
      const float* piece0 = p.ws + (size_t)piece_slot(p.iters, G, ga + 1, tile_begin) * (C::TM * BN);
      const size_t piece_stride = 2 * (size_t)(C::TM * BN);  // slot 2g of consecutive CTAs
      auto chunk_floats = [](int ch) { return ((ch / C::CHUNKS) * (BN / 4) + (ch % C::CHUNKS) * 8) * BM * 4; };
      auto chunk_bytes = [](int ch) { return BM * 16 * min(8, BN / 4 - (ch % C::CHUNKS) * 8); };
      if (batch >= 1) {
        auto issue = [&](int b0, int half) {
          uint32_t bytes = 0;
          for (int ch = b0; ch < b0 + batch && ch < kTotalChunks; ++ch) bytes += (uint32_t)(others * chunk_bytes(ch));
          mbar_arrive_expect_tx(&fbar[half], bytes);
          for (int ch = b0; ch < b0 + batch && ch < kTotalChunks; ++ch)
            for (int pi = 0; pi < others; ++pi)
              bulk_load(smem + half * kHalf + ((ch - b0) * others + pi) * kChunkBytes,
                        piece0 + pi * piece_stride + chunk_floats(ch), (uint32_t)chunk_bytes(ch), &fbar[half]);
        };
        const int nbatch = (kTotalChunks + batch - 1) / batch;
        int issued = 0;  // batches issued (tracked by et == 0)
        if (et == 0) {
          issue(0, 0);
          issued = 1;
          if (nbatch > 1) {
            issue(batch, 1);
            issued = 2;
          }
        }
        int bi = 0;
        for (int b0 = 0; b0 < kTotalChunks; b0 += batch, ++bi) {
          const int half = bi & 1;
          if (et == 0) *s_flag = wait_or_abort(&fbar[half], (uint32_t)((bi >> 1) & 1), p.status, s_abort) ? 1 : 0;
          epi_bar();
          if (!*s_flag) {
            // no bulk copy may still be in flight when the CTA exits (bounded waits)
            if (et == 0)
              for (int bj = bi; bj < issued; ++bj) mbar_wait(&fbar[bj & 1], (uint32_t)((bj >> 1) & 1), p.status);
            break;
          }
#pragma unroll 1
          for (int ch = b0; ch < b0 + batch && ch < kTotalChunks; ++ch, ++emitted) {
            const int w = ch / C::CHUNKS, c = ch % C::CHUNKS;
            float v[32];
            tmem_ld32(taddr + w * C::ACC_STRIDE + c * 32, v);
            for (int pi = 0; pi < others; ++pi) {
              const float4* src = reinterpret_cast<const float4*>(smem + half * kHalf + ((ch - b0) * others + pi) * kChunkBytes);
#pragma unroll
              for (int j4 = 0; j4 < 8; ++j4)
                if (c * 32 + j4 * 4 < BN) {
                  const float4 x = src[j4 * BM + row];
                  v[4 * j4] += x.x;
                  v[4 * j4 + 1] += x.y;
                  v[4 * j4 + 2] += x.z;
                  v[4 * j4 + 3] += x.w;
                }
            }
            emit_chunk<BN, EPI>(p, v, wt * C::TM + w * BM, row, mbase + c * 32, c * 32, lane, q, et,
                                stg + (emitted & 1) * kStgBytes, s_keys, s_best);
          }
          epi_bar();  // every thread is done with this half before it is refilled
          if (et == 0 && bi + 2 < nbatch) {
            issue(b0 + 2 * batch, half);
            ++issued;
          }
        }
      } else {
        // too many pieces for the ring: read them straight from the workspace
        __threadfence();
#pragma unroll 1
        for (int ch = 0; ch < kTotalChunks; ++ch, ++emitted) {
          const int w = ch / C::CHUNKS, c = ch % C::CHUNKS;
          float v[32];
          tmem_ld32(taddr + w * C::ACC_STRIDE + c * 32, v);
          for (int pi = 0; pi < others; ++pi) {
            const float4* src = reinterpret_cast<const float4*>(piece0 + pi * piece_stride + chunk_floats(ch));
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4)
              if (c * 32 + j4 * 4 < BN) {
                const float4 x = ld_cg_f4(src + j4 * BM + row);
                v[4 * j4] += x.x;
                v[4 * j4 + 1] += x.y;
                v[4 * j4 + 2] += x.z;
                v[4 * j4 + 3] += x.w;
              }
          }
          emit_chunk<BN, EPI>(p, v, wt * C::TM + w * BM, row, mbase + c * 32, c * 32, lane, q, et,
                              stg + (emitted & 1) * kStgBytes, s_keys, s_best);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&aempty[buf]);
    }
    if constexpr (EPI == 2) {
      if (best_tt >= 0) flush_keys<BN>(p, s_best, best_tt * BN, et);
      // Every CTA counts itself done after its last key update; the last one writes the ids.
      __threadfence();
      epi_bar();
      if (et == 0) *s_flag = atomicAdd(p.done, 1) == G - 1;
      epi_bar();
      if (*s_flag) {
        __threadfence();
        for (int m = et; m < p.M; m += kEpiThreads) {
          const unsigned long long k = atomicExch(p.keys + m, 0ull);
          const int64_t id = (int64_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
          const int orow = p.out_rows ? p.out_rows[m] : m;
          if (orow >= 0) p.out_ids[orow] = id;
          if (p.token_rows != nullptr && p.token_rows[m] >= 0) p.token_table[p.token_rows[m]] = (int32_t)id;
        }
        if (et == 0) atomicExch(p.done, 0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encoder() {
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

struct Key {
  const void* ptr;
  int64_t rows, cols, ld;
  int box_rows;
  bool operator==(const Key& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows;
  }
};
struct KeyHash {
  size_t operator()(const Key& k) const {
    return std::hash<const void*>()(k.ptr) ^ (std::hash<int64_t>()(k.rows) * 31) ^ (std::hash<int64_t>()(k.cols) * 131) ^
           (std::hash<int64_t>()(k.ld) * 1313) ^ ((size_t)k.box_rows << 40);
  }
};

// 2-D row-major bf16 matrix [rows, cols] with leading dimension ld, tile box {64 cols, box_rows}.
static int matrix_map(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, KeyHash> cache;
  const Key key{ptr, rows, cols, ld, box_rows};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return CDB_OK;
  }
  EncodeFn enc = encoder();
  if (enc == nullptr) return CDB_ERR_TMA_ENCODE;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return CDB_ERR_TMA_ENCODE;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, map);
  *out = map;
  return CDB_OK;
}

template <int BN, int EPI, int WM>
static int launch(const CUtensorMap& mw, const CUtensorMap& mx, const Params& p, int ctas, cudaStream_t st) {
  using C = Cfg<BN, WM>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(gemm_kernel<BN, EPI, WM>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return CDB_ERR_CUDA;
    attr_set = true;
  }
  prefer_max_shared(reinterpret_cast<const void*>(gemm_kernel<BN, EPI, WM>));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_kernel<BN, EPI, WM>, mw, mx, p) == cudaSuccess ? CDB_OK : CDB_ERR_CUDA;
}

// Token-tile width for M token rows: M rounded up to a multiple of 16 (the UMMA N step for
// M = 128) up to 256; wider problems tile the tokens by 256.
static int tile_n_for(int M) { return M >= 256 ? 256 : ((M + 15) / 16) * 16; }

struct Shape {
  int bn, wm, tiles_w, tiles_tok, kb, ctas;
  long long iters;
};

// Problems with more than one 256-token tile (prefill) take 256 x 256 tiles (two weight tiles
// per CTA tile) for the plain and argmax epilogues; decode-sized ones, and the SwiGLU epilogue
// (whose arithmetic must overlap the next tile's main loop, which needs two accumulator
// buffers), 128 weight rows per tile.
static Shape shape_for(int M, int N, int K, int max_ctas, int num_sms, int epi = 0) {
  Shape s;
  s.bn = tile_n_for(M);
  s.wm = M > 256 && epi != 1 ? 2 : 1;
  s.tiles_w = (N + s.wm * BM - 1) / (s.wm * BM);
  s.tiles_tok = (M + s.bn - 1) / s.bn;
  s.kb = (K + BK - 1) / BK;
  s.iters = (long long)s.tiles_w * s.tiles_tok * s.kb;
  int g = (num_sms > 0 ? num_sms : 148) * (s.bn < 128 ? 2 : 1);  // narrow token tiles: two CTAs per SM
  if (max_ctas > 0 && max_ctas < g) g = max_ctas;
  s.ctas = (int)(s.iters < g ? s.iters : g);
  return s;
}

#include "gemm_cluster.cuh"
#include "gemm_pair.cuh"

// Split mode (gemm_cluster.cuh) when the tiles cannot fill the SMs (EPI 0 and 1; the LM head
// always has more tiles), stream-K otherwise.
template <int BN, int EPI>
static int dispatch(const CUtensorMap& mw, const CUtensorMap& mx, const Params& p, const struct Shape& s, int num_sms,
                    bool split, cudaStream_t st) {
  if constexpr (EPI != 2) {
    if (split) {
      cl::CParams c;
      c.c = p.c;
      c.ldc = p.ldc;
      c.M = p.M;
      c.N = p.N;
      c.K = p.K;
      c.splits = 1;
      c.kb_per_split = p.kb;
      c.num_kb = p.kb;
      c.vec_store = p.vec_store;
      c.status = p.status;
      return cl::launch_cluster<BN, EPI>(mw, mx, c, (p.N + BM - 1) / BM, s.tiles_tok, num_sms, st);
    }
  }
  if constexpr (BN == 256) {
    if (s.wm == 2) return launch<BN, EPI, 2>(mw, mx, p, s.ctas, st);
  }
  return launch<BN, EPI, 1>(mw, mx, p, s.ctas, st);
}

// Shared host path of the three epilogues: c = epilogue(x[M,K] * w[N,K]^T).
template <int EPI>
static int run(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int M, int N, int K,
               int max_ctas, float* workspace, int64_t workspace_elems, int32_t* counters, int num_counters,
               int num_sms, int32_t* status, cudaStream_t st, const Params* epi2 = nullptr) {
  if (K % 8 != 0 || ldx % 8 != 0 || ldw % 8 != 0 || ldx < K || ldw < K) return CDB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) return CDB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(workspace) & 15)) return CDB_ERR_INVALID_ARGUMENT;
  const Shape s = shape_for(M, N, K, max_ctas, num_sms, EPI);
  if ((long long)s.tiles_w * s.tiles_tok > num_counters || counters == nullptr) return CDB_ERR_INVALID_ARGUMENT;
  if ((int64_t)2 * s.ctas * s.wm * BM * s.bn > workspace_elems || workspace == nullptr) return CDB_ERR_INVALID_ARGUMENT;
  CUtensorMap mw, mx;
  int rc = matrix_map(&mw, w, N, K, ldw, BM);
  if (rc != CDB_OK) return rc;
  rc = matrix_map(&mx, x, M, K, ldx, s.bn);
  if (rc != CDB_OK) return rc;
  Params p;
  std::memset(&p, 0, sizeof(p));
  p.c = static_cast<__nv_bfloat16*>(c);
  p.ldc = ldc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.tiles_w = s.tiles_w;
  p.tiles_tok = s.tiles_tok;
  p.kb = s.kb;
  p.iters = s.iters;
  p.ws = workspace;
  p.ctr = counters;
  p.pair_store = ((reinterpret_cast<uintptr_t>(c) & 3) == 0 && ldc % 2 == 0 && N % 2 == 0) ? 1 : 0;
  p.vec_store = ((reinterpret_cast<uintptr_t>(c) & 7) == 0 && ldc % 4 == 0) ? 1 : 0;
  p.vec16 = ((reinterpret_cast<uintptr_t>(c) & 15) == 0 && ldc % 8 == 0) ? 1 : 0;
  p.status = status;
  const int sms = num_sms > 0 ? num_sms : 148;
  // split mode for problems with fewer tiles than SMs; the SwiGLU epilogue there pairs 4 rows
  const long long tiles128 = (long long)((N + BM - 1) / BM) * s.tiles_tok;
  const bool split = EPI != 2 && max_ctas <= 0 && tiles128 < sms && (EPI != 1 || N % 4 == 0);
  // Prefill-shaped problems (more than 256 token rows) with the plain and SwiGLU epilogues run on
  // CTA pairs (gemm_pair.cuh) when there are at least two pair tiles per pair (below that the
  // double-buffered accumulators have nothing to overlap, and the one-SM stream-K measured faster:
  // 32.8 against 36.9 us at 600 x 6144 x 2048) and the counters, workspace and resident clusters
  // allow it.
  if constexpr (EPI != 2) {
    if (M > 256 && max_ctas <= 0) {
      const int tiles_w2 = (N + pair::PTM - 1) / pair::PTM;
      const long long tiles2 = (long long)tiles_w2 * s.tiles_tok;
      const long long iters2 = tiles2 * s.kb;
      long long pairs = sms / 2;
      const int resident = pair::max_resident_pairs<EPI>();
      if (resident < pairs) pairs = resident;
      if (iters2 < pairs) pairs = iters2;
      if (pairs >= 1 && tiles2 >= 2 * pairs && 2 * tiles2 <= num_counters &&
          4LL * pairs * BM * pair::PBN <= workspace_elems) {
        CUtensorMap mx_half;
        rc = matrix_map(&mx_half, x, M, K, ldx, pair::HALF_ROWS);
        if (rc != CDB_OK) return rc;
        p.tiles_w = tiles_w2;
        p.iters = iters2;
        return pair::launch_pair<EPI>(mw, mx_half, p, (int)pairs, st);
      }
    }
  }
  if (epi2 != nullptr) {
    p.keys = epi2->keys;
    p.done = epi2->done;
    p.out_ids = epi2->out_ids;
    p.out_rows = epi2->out_rows;
    p.token_rows = epi2->token_rows;
    p.token_table = epi2->token_table;
  }
  switch (s.bn) {
#define CDB_GEMM_CASE(B) \
  case B:                \
    return dispatch<B, EPI>(mw, mx, p, s, sms, split, st);
    CDB_GEMM_CASE(16)
    CDB_GEMM_CASE(32)
    CDB_GEMM_CASE(48)
    CDB_GEMM_CASE(64)
    CDB_GEMM_CASE(80)
    CDB_GEMM_CASE(96)
    CDB_GEMM_CASE(112)
    CDB_GEMM_CASE(128)
    CDB_GEMM_CASE(144)
    CDB_GEMM_CASE(160)
    CDB_GEMM_CASE(176)
    CDB_GEMM_CASE(192)
    CDB_GEMM_CASE(208)
    CDB_GEMM_CASE(224)
    CDB_GEMM_CASE(240)
    CDB_GEMM_CASE(256)
#undef CDB_GEMM_CASE
    default:
      return CDB_ERR_UNSUPPORTED;
  }
}

}  // namespace gemm
}  // namespace cdb

extern "C" int cdb_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int M,
                             int N, int K, int max_ctas, float* workspace, int64_t workspace_elems, int32_t* counters,
                             int num_counters, int num_sms, int32_t* status, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0) return M == 0 ? CDB_OK : CDB_ERR_INVALID_ARGUMENT;
  if (ldc < N) return CDB_ERR_INVALID_ARGUMENT;
  return cdb::gemm::run<0>(x, ldx, w, ldw, c, ldc, M, N, K, max_ctas, workspace, workspace_elems, counters,
                           num_counters, num_sms, status, static_cast<cudaStream_t>(stream));
}

extern "C" int cdb_mlp_gateup_silu_gemm(const void* x, int64_t ldx, const void* w_gate_up, int64_t ldw, void* act,
                                        int64_t ld_act, int M, int inter, int K, int max_ctas, float* workspace,
                                        int64_t workspace_elems, int32_t* counters, int num_counters, int num_sms,
                                        int32_t* status, void* stream) {
  if (M <= 0 || inter <= 0 || K <= 0) return M == 0 ? CDB_OK : CDB_ERR_INVALID_ARGUMENT;
  if (ld_act < inter || (reinterpret_cast<uintptr_t>(act) & 1)) return CDB_ERR_INVALID_ARGUMENT;
  return cdb::gemm::run<1>(x, ldx, w_gate_up, ldw, act, ld_act, M, 2 * inter, K, max_ctas, workspace,
                           workspace_elems, counters, num_counters, num_sms, status, static_cast<cudaStream_t>(stream));
}

extern "C" int cdb_lm_head_argmax(const void* x, int64_t ldx, const void* w, int64_t ldw, int M, int vocab, int K,
                                  int64_t* out_ids, const int32_t* out_rows, const int32_t* token_rows,
                                  int32_t* token_table, uint64_t* keys, int32_t* done, float* workspace,
                                  int64_t workspace_elems, int32_t* counters, int num_counters, int num_sms,
                                  int32_t* status, void* stream) {
  if (M <= 0 || vocab <= 0 || K <= 0) return M == 0 ? CDB_OK : CDB_ERR_INVALID_ARGUMENT;
  if (out_ids == nullptr || keys == nullptr || done == nullptr || (token_rows != nullptr && token_table == nullptr))
    return CDB_ERR_INVALID_ARGUMENT;
  cdb::gemm::Params e;
  std::memset(&e, 0, sizeof(e));
  e.keys = reinterpret_cast<unsigned long long*>(keys);
  e.done = done;
  e.out_ids = out_ids;
  e.out_rows = out_rows;
  e.token_rows = token_rows;
  e.token_table = token_table;
  return cdb::gemm::run<2>(x, ldx, w, ldw, nullptr, 0, M, vocab, K, 0, workspace, workspace_elems, counters,
                           num_counters, num_sms, status, static_cast<cudaStream_t>(stream), &e);
}

namespace cdb {
namespace gemm {
static int run_partials(const void* x, int64_t ldx, const void* w, int64_t ldw, float* parts, int64_t part_stride,
                        int M, int N, int K, int splits, int32_t* status, cudaStream_t st) {
  if (K % 8 != 0 || ldx % 8 != 0 || ldw % 8 != 0 || ldx < K || ldw < K) return CDB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) return CDB_ERR_INVALID_ARGUMENT;
  if (parts == nullptr || (reinterpret_cast<uintptr_t>(parts) & 3) || part_stride < (int64_t)M * N) return CDB_ERR_INVALID_ARGUMENT;
  const int bn = tile_n_for(M);
  const int num_kb = (K + BK - 1) / BK;
  if (splits < 1 || splits > cl::kMaxPartSplits || splits > num_kb) return CDB_ERR_INVALID_ARGUMENT;
  CUtensorMap mw, mx;
  int rc = matrix_map(&mw, w, N, K, ldw, BM);
  if (rc != CDB_OK) return rc;
  rc = matrix_map(&mx, x, M, K, ldx, bn);
  if (rc != CDB_OK) return rc;
  cl::CParams c;
  std::memset(&c, 0, sizeof(c));
  c.M = M;
  c.N = N;
  c.K = K;
  c.splits = splits;
  c.num_kb = num_kb;
  c.status = status;
  c.parts = parts;
  c.part_stride = part_stride;
  const int tiles_n = (N + BM - 1) / BM, tiles_m = (M + bn - 1) / bn;
  switch (bn) {
#define CDB_PART_CASE(B) \
  case B:                \
    return cl::launch_partials<B>(mw, mx, c, tiles_n, tiles_m, st);
    CDB_PART_CASE(16)
    CDB_PART_CASE(32)
    CDB_PART_CASE(48)
    CDB_PART_CASE(64)
    CDB_PART_CASE(80)
    CDB_PART_CASE(96)
    CDB_PART_CASE(112)
    CDB_PART_CASE(128)
    CDB_PART_CASE(144)
    CDB_PART_CASE(160)
    CDB_PART_CASE(176)
    CDB_PART_CASE(192)
    CDB_PART_CASE(208)
    CDB_PART_CASE(224)
    CDB_PART_CASE(240)
    CDB_PART_CASE(256)
#undef CDB_PART_CASE
    default:
      return CDB_ERR_UNSUPPORTED;
  }
}
}  // namespace gemm
}  // namespace cdb

extern "C" int cdb_gemm_partial_splits(int M, int N, int K, int num_sms) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int bn = cdb::gemm::tile_n_for(M);
  const int tiles = ((N + cdb::gemm::BM - 1) / cdb::gemm::BM) * ((M + bn - 1) / bn);
  return cdb::gemm::cl::partial_splits(bn, tiles, (K + cdb::gemm::BK - 1) / cdb::gemm::BK, num_sms > 0 ? num_sms : 148);
}

extern "C" int cdb_gemm_bf16_partials(const void* x, int64_t ldx, const void* w, int64_t ldw, float* parts,
                                      int64_t part_stride, int M, int N, int K, int splits, int32_t* status,
                                      void* stream) {
  if (M <= 0 || N <= 0 || K <= 0) return M == 0 ? CDB_OK : CDB_ERR_INVALID_ARGUMENT;
  return cdb::gemm::run_partials(x, ldx, w, ldw, parts, part_stride, M, N, K, splits, status,
                                 static_cast<cudaStream_t>(stream));
}

extern "C" int64_t cdb_gemm_workspace_elems(int M, int N, int K, int num_sms) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const cdb::gemm::Shape s = cdb::gemm::shape_for(M, N, K, 0, num_sms);
  return (int64_t)2 * s.ctas * s.wm * cdb::gemm::BM * s.bn;
}

extern "C" int cdb_gemm_counter_elems(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const cdb::gemm::Shape s = cdb::gemm::shape_for(M, N, K, 0, 148, 1);  // 128-row tiles: the most tiles
  return s.tiles_w * s.tiles_tok;
}
