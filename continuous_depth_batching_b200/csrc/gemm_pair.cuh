// Pair mode of the stream-K GEMM (included by gemm.cu inside namespace cdb::gemm, after the
// stream-K helpers it shares): prefill-shaped problems (more than 256 token rows, plain and SwiGLU
// epilogues) on CTA pairs that issue tcgen05.mma.cta_group::2.
//
// A pair tile is 256 weight rows x 256 tokens. The two CTAs of a 2-CTA cluster each stage half of
// it per 64-wide k block, 32 KB per stage: CTA r loads weight rows [256 wt + 128 r, +128) (its half
// of UMMA A, M = 256) and tokens [256 tt + 128 r, +128) (its half of UMMA B, N = 256). One thread
// of the even CTA (the leader) issues M = 256, N = 256 MMAs that read both CTAs' stages and leave
// weight rows 128 r .. 128 r + 127 of the fp32 accumulator in CTA r's tensor memory: 256 columns
// per CTA, so each CTA holds two accumulator buffers and a tile's epilogue overlaps the next
// tile's main loop. Per FLOP a pair fills as many shared-memory bytes as the one-SM 256 x 256
// tile, which needs all 512 TMEM columns of its SM for one accumulator and so runs its epilogue
// between tiles.
//
// Signalling: both CTAs' TMA loads complete on the leader's `full` barrier (the .cta_group::2
// load form, the barrier addressed in the leader's shared memory through mapa); the leader's
// commits arrive on `empty`, `afull` and `mdrain` of both CTAs (tcgen05.commit with a CTA mask);
// both CTAs' epilogue warps arrive on the leader's `aempty` (8 arrivals per buffer and tile). Every
// TMA load fills only the issuing CTA's own shared memory.
//
// Work split: stream-K over pairs - the pair index in place of the CTA index of the one-SM kernel -
// with its owner fixup done per half: CTA r of a pair publishes and combines only its own 128
// weight rows, in workspace slot 2 * slot + r and tile counter 2 t + r. Every pair of a launch is
// co-resident (the host caps the pairs at cudaOccupancyMaxActiveClusters), as owners wait on later
// pairs' pieces. (Data-parallel waves of whole tiles first, pair g taking tiles g, g + G, ..., with
// stream-K only for the remainder, measured 15-28% slower at the 8192-token projections: the pairs
// of a wave all read the same few token and weight tiles at once.)
//
// Warp roles (192 threads, the same in both CTAs): warp 0 TMA producer; warp 1 allocates TMEM
// (cta_group::2, both CTAs) and, in the leader, issues the MMAs; warps 2..5 epilogue.
#pragma once

namespace pair {

constexpr int PBN = 256;              // tokens of a pair tile
constexpr int PTM = 2 * BM;           // weight rows of a pair tile
constexpr int HALF_ROWS = 128;        // tokens (and weight rows) one CTA stages
constexpr int A_BYTES = BM * BK * 2;  // this CTA's 128 weight rows of one k block
constexpr int B_BYTES = HALF_ROWS * BK * 2;
constexpr int STAGE = A_BYTES + B_BYTES;
constexpr int STAGES = 6;
constexpr int THREADS_P = 6 * 32;
constexpr int kWarpProd = 0, kWarpMmaP = 1;
constexpr int ACC_COLS = PBN;  // one buffer: 128 lanes x 256 fp32 columns
constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
constexpr int OFF_BAR = STAGES * STAGE;
constexpr int NBAR = 2 * STAGES + 2 + 2 + 1 + 2;  // full, empty, afull[2], aempty[2], mdrain, fbar[2]
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int OFF_STG = (OFF_MISC + 64 + 15) / 16 * 16;  // 2 staging tiles
constexpr int SMEM = OFF_STG + 2 * kStgBytes + 1024;     // + alignment slack
// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, M = 256 (the
// pair's weight rows), N = 256.
constexpr uint32_t IDESC =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PBN >> 3) << 17) | ((uint32_t)(PTM >> 4) << 24);
static_assert(STAGE % 1024 == 0 && A_BYTES % 1024 == 0, "swizzled stages stay 1024-byte aligned");
static_assert(SMEM <= 227 * 1024, "shared memory");
static_assert(OFF_BAR / 2 >= BM * 32 * 4, "a fixup batch (half the ring) holds at least one 32-token chunk");

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
// Shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// 2-D tile load into this CTA's shared memory that completes on a barrier of either CTA of the
// pair (`bar` is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// wait_or_abort for a barrier that the other CTA of the pair also arrives on
__device__ __forceinline__ bool wait_or_abort_cluster(uint64_t* bar, uint32_t parity, int32_t* status,
                                                      volatile int* abort) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort) return false;
  }
  set_error(status, CDB_ERR_DEVICE_TIMEOUT);
  *abort = 1;
  return false;
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_pair_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once, when every MMA issued so far has completed) on `bar` in both CTAs of the pair.
__device__ __forceinline__ void umma_pair_commit(uint64_t* bar) {
  const uint16_t both = 3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(both)
      : "memory");
}

// A pair's work: its stream-K range [it0, it1) of the (tile, 64-wide k block) iterations, tiles
// in token-major order. The pair's k blocks are numbered 0 .. n-1; block i uses ring stage
// i % STAGES. The host launches at most `iters` pairs, so no range is empty (an owner counts every
// pair between it and the tile's last piece as a piece).
struct PairWork {
  int kb;
  long long iters, it0, it1, n;

  __device__ PairWork(int tiles, int kb_, int G, int g) : kb(kb_) {
    iters = (long long)tiles * kb;
    it0 = range_start(iters, G, g);
    it1 = range_start(iters, G, g + 1);
    n = it1 - it0;
  }
  // tile and k block of this pair's block i
  __device__ void at(long long i, int& t, int& k) const {
    const long long it = it0 + i;
    t = (int)(it / kb);
    k = (int)(it % kb);
  }
  // end (exclusive) of the segment - one tile's run of k blocks - that starts at block i
  __device__ long long seg_end(long long i) const {
    const long long e = ((it0 + i) / kb + 1) * kb;
    return (e < it1 ? e : it1) - it0;
  }
};

template <int EPI>
__global__ void __launch_bounds__(THREADS_P, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);  // used in the leader only
  uint64_t* empty = full + STAGES;
  uint64_t* afull = empty + STAGES;
  uint64_t* aempty = afull + 2;  // used in the leader only
  uint64_t* mdrain = aempty + 2;
  uint64_t* fbar = mdrain + 1;  // [2] owner fixup: bulk copies of the other pieces
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);
  volatile int* s_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 16);
  uint8_t* stg = smem + OFF_STG;
  cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = (int)cluster_ctarank();
  const bool leader = rank == 0;
  const int G = (int)(gridDim.x >> 1);  // pairs
  const int g = (int)cluster_id_x();    // this pair
  const int kb = p.kb;
  const PairWork work(p.tiles_w * p.tiles_tok, kb, G, g);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);  // the leader's expect_tx; both CTAs' bytes
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&afull[b], 1);
      mbar_init(&aempty[b], 8);  // four epilogue warps of each CTA
    }
    mbar_init(mdrain, 1);
    mbar_init(&fbar[0], 1);
    mbar_init(&fbar[1], 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMmaP) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Both CTAs' barriers are initialised and both TMEM allocations made before any signal or MMA
  // crosses to the other CTA.
  cluster.sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == kWarpProd) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tensormap(&map_w);
      prefetch_tensormap(&map_x);
      const uint32_t full_leader = map_rank(smem_u32(full), 0);
      const long long n = work.n;
      const long long npre = n < STAGES ? n : STAGES;
      int t, k;
      // the weight tiles of the first stages before the predecessor is waited for
      for (long long i = 0; i < npre; ++i) {
        work.at(i, t, k);
        if (leader) mbar_arrive_expect_tx(&full[i], 2 * STAGE);
        tma_load_2d_pair(smem + i * STAGE, &map_w, full_leader + (uint32_t)(i * 8), k * BK,
                         (t % p.tiles_w) * PTM + rank * BM);
      }
      pdl_wait();
      for (long long i = 0; i < npre; ++i) {
        work.at(i, t, k);
        tma_load_2d_pair(smem + i * STAGE + A_BYTES, &map_x, full_leader + (uint32_t)(i * 8), k * BK,
                         (t / p.tiles_w) * PBN + rank * HALF_ROWS);
      }
      long long i = npre;
      for (; i < n; ++i) {
        work.at(i, t, k);
        const int s = (int)(i % STAGES);
        if (!wait_or_abort(&empty[s], (uint32_t)(((i / STAGES) & 1) ^ 1), p.status, s_abort)) break;
        if (leader) mbar_arrive_expect_tx(&full[s], 2 * STAGE);
        tma_load_2d_pair(smem + s * STAGE, &map_w, full_leader + (uint32_t)(s * 8), k * BK,
                         (t % p.tiles_w) * PTM + rank * BM);
        tma_load_2d_pair(smem + s * STAGE + A_BYTES, &map_x, full_leader + (uint32_t)(s * 8), k * BK,
                         (t / p.tiles_w) * PBN + rank * HALF_ROWS);
      }
      // No copy may still be in flight when the CTAs exit. Both CTAs' copies complete on the
      // leader's barriers, which the leader waits for (bounded); the closing cluster barrier keeps
      // the other CTA alive until then.
      if (leader)
        for (long long j = (i > STAGES ? i - STAGES : 0); j < i; ++j)
          mbar_wait(&full[j % STAGES], (uint32_t)((j / STAGES) & 1), p.status);
    }
    __syncwarp();  // the warp reaches the closing barriers converged
  } else if (warp == kWarpMmaP) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      long long i = 0;
      int seg = 0;
      bool ok = true;
      for (; i < work.n && ok; ++seg) {
        const long long seg_end = work.seg_end(i);
        const int buf = seg & 1;
        if (!wait_or_abort_cluster(&aempty[buf], (uint32_t)(((seg >> 1) & 1) ^ 1), p.status, s_abort)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * ACC_COLS);
        for (bool first = true; i < seg_end; ++i, first = false) {
          const int s = (int)(i % STAGES);
          if (!wait_or_abort(&full[s], (uint32_t)((i / STAGES) & 1), p.status, s_abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * STAGE);
          const uint32_t b = a + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_pair_bf16(d, sw128_desc(a + kk * 32), sw128_desc(b + kk * 32), IDESC, (!first || kk > 0) ? 1u : 0u);
          umma_pair_commit(&empty[s]);
        }
        if (ok) umma_pair_commit(&afull[buf]);
      }
      // On every path (an abandoned wait included) both CTAs learn when no MMA runs any more.
      umma_pair_commit(mdrain);
    }
    // Both CTAs: every MMA - which reads both CTAs' stages and writes both CTAs' TMEM - has
    // completed before either CTA frees TMEM or exits.
    if (lane == 0) mbar_wait(mdrain, 0, p.status);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int et = threadIdx.x - 64;
    const int row = q * 32 + lane;
    const uint32_t aempty_leader = map_rank(smem_u32(aempty), 0);
    pdl_wait();  // outputs, workspace and counters may still be in use by the predecessor
    int seg = 0, emitted = 0;
    for (long long i = 0; i < work.n; ++seg) {
      const long long e = work.seg_end(i);
      int t, k0;
      work.at(i, t, k0);
      const bool whole = k0 == 0 && e - i == kb;  // the segment holds all of its tile's k blocks
      const long long tile_begin = (long long)t * kb;
      i = e;
      const int buf = seg & 1;
      if (et == 0) *s_flag = wait_or_abort(&afull[buf], (uint32_t)((seg >> 1) & 1), p.status, s_abort) ? 1 : 0;
      epi_bar();
      if (!*s_flag) break;
      epi_bar();  // everyone has read the flag before it is reused
      tc_fence_after();
      const int wt = t % p.tiles_w, tt = t / p.tiles_w;
      const int n0 = wt * PTM + rank * BM;  // this CTA's weight rows
      const int mbase = tt * PBN;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * ACC_COLS);
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(aempty_leader + (uint32_t)(buf * 8));
      };
      if (whole) {
#pragma unroll 1
        for (int c = 0; c < PBN / 32; ++c, ++emitted) {
          float v[32];
          tmem_ld32(taddr + c * 32, v);
          emit_chunk<PBN, EPI>(p, v, n0, row, mbase + c * 32, c * 32, lane, q, et, stg + (emitted & 1) * kStgBytes,
                               nullptr, nullptr);
        }
        release();
        continue;
      }
      // Split tile: as in the one-SM kernel, per half. The owner pair holds the tile's first k
      // block (its range's last segment); the other pieces are first segments of later pairs.
      const int ga = cta_of(work.iters, G, tile_begin);
      const int gb = cta_of(work.iters, G, tile_begin + kb - 1);
      constexpr int kPiece = BM * PBN;  // floats of one half piece
      if (g != ga) {
        float4* mine =
            reinterpret_cast<float4*>(p.ws + ((size_t)piece_slot(work.iters, G, g, tile_begin) * 2 + rank) * kPiece);
#pragma unroll 1
        for (int c = 0; c < PBN / 32; ++c) {
          float v[32];
          tmem_ld32(taddr + c * 32, v);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            mine[(c * 8 + j4) * BM + row] = make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
        }
        release();
        __threadfence();
        epi_bar();
        if (et == 0) atomicAdd(p.ctr + 2 * t + rank, 1);
        continue;
      }
      // Owner half: wait until the other gb - ga pieces of this half are published, then add them
      // in pair order to the accumulator (the same order in every run). This CTA's ring is idle
      // (the range's last segment, every MMA completed), so the pieces come in by bulk copies,
      // double-buffered in batches of 32-token chunks.
      const int others = gb - ga;
      if (et == 0) {
        bool ok = false;
        for (uint32_t w = 0; w < (kSpinLimit >> 4); ++w) {
          if (ld_acquire(p.ctr + 2 * t + rank) >= others) {
            ok = true;
            break;
          }
          if (*s_abort) break;
          __nanosleep(64);
        }
        if (ok) {
          p.ctr[2 * t + rank] = 0;  // every piece has arrived: ready for the next call
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
      constexpr int kChunkBytes = BM * 32 * 4;  // one 32-token chunk of a half piece
      constexpr int kHalfRing = OFF_BAR / 2;
      constexpr int kTotalChunks = PBN / 32;
      const int batch = kHalfRing / (others * kChunkBytes);
      const float* piece0 = p.ws + ((size_t)piece_slot(work.iters, G, ga + 1, tile_begin) * 2 + rank) * kPiece;
      const size_t piece_stride = 4 * (size_t)kPiece;  // slot 2g of consecutive pairs, this half
      if (batch >= 1) {
        auto issue = [&](int b0, int half) {
          const int nch = min(batch, kTotalChunks - b0);
          mbar_arrive_expect_tx(&fbar[half], (uint32_t)(nch * others * kChunkBytes));
          for (int ch = b0; ch < b0 + nch; ++ch)
            for (int pi = 0; pi < others; ++pi)
              bulk_load(smem + half * kHalfRing + ((ch - b0) * others + pi) * kChunkBytes,
                        piece0 + pi * piece_stride + (size_t)ch * 8 * BM * 4, (uint32_t)kChunkBytes, &fbar[half]);
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
            float v[32];
            tmem_ld32(taddr + ch * 32, v);
            for (int pi = 0; pi < others; ++pi) {
              const float4* src =
                  reinterpret_cast<const float4*>(smem + half * kHalfRing + ((ch - b0) * others + pi) * kChunkBytes);
#pragma unroll
              for (int j4 = 0; j4 < 8; ++j4) {
                const float4 x = src[j4 * BM + row];
                v[4 * j4] += x.x;
                v[4 * j4 + 1] += x.y;
                v[4 * j4 + 2] += x.z;
                v[4 * j4 + 3] += x.w;
              }
            }
            emit_chunk<PBN, EPI>(p, v, n0, row, mbase + ch * 32, ch * 32, lane, q, et,
                                 stg + (emitted & 1) * kStgBytes, nullptr, nullptr);
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
          float v[32];
          tmem_ld32(taddr + ch * 32, v);
          for (int pi = 0; pi < others; ++pi) {
            const float4* src = reinterpret_cast<const float4*>(piece0 + pi * piece_stride + (size_t)ch * 8 * BM * 4);
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 x = ld_cg_f4(src + j4 * BM + row);
              v[4 * j4] += x.x;
              v[4 * j4 + 1] += x.y;
              v[4 * j4 + 2] += x.z;
              v[4 * j4 + 3] += x.w;
            }
          }
          emit_chunk<PBN, EPI>(p, v, n0, row, mbase + ch * 32, ch * 32, lane, q, et, stg + (emitted & 1) * kStgBytes,
                               nullptr, nullptr);
        }
      }
      release();
    }
  }
  tc_fence_before();
  // Neither CTA frees TMEM or exits while the other may still signal its barriers, read its
  // stages (the leader's MMAs) or have copies landing (the leader's barriers).
  cluster.sync();
  if (warp == kWarpMmaP) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side of the pair mode
static cudaLaunchConfig_t pair_config(dim3 grid, cudaStream_t st, cudaLaunchAttribute (&attr)[2]) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(THREADS_P);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cfg;
}

// Pairs that can be resident at once (0 if the attribute or the query fails).
template <int EPI>
static int max_resident_pairs() {
  static std::mutex mu;
  static int cached = -1;
  std::lock_guard<std::mutex> lock(mu);
  if (cached < 0) {
    cached = 0;
    if (cudaFuncSetAttribute(gemm_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) == cudaSuccess) {
      prefer_max_shared(reinterpret_cast<const void*>(gemm_pair_kernel<EPI>));
      cudaLaunchAttribute attr[2];
      cudaLaunchConfig_t cfg = pair_config(dim3(2), nullptr, attr);
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<EPI>, &cfg) == cudaSuccess) cached = n;
    }
    cudaGetLastError();
  }
  return cached;
}

template <int EPI>
static int launch_pair(const CUtensorMap& mw, const CUtensorMap& mx, const Params& p, int pairs, cudaStream_t st) {
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = pair_config(dim3(2 * pairs), st, attr);
  return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<EPI>, mw, mx, p) == cudaSuccess ? CDB_OK : CDB_ERR_CUDA;
}

}  // namespace pair
