// Split mode of the tcgen05 GEMM (included by gemm.cu inside namespace cdb::gemm, after the
// shared helpers it uses): the
// K range of every output tile is split over one thread-block cluster (grid z = cluster z =
// splits <= 8). It serves problems with fewer output tiles than SMs - every decode-shaped
// projection - where stream-K would cut each tile into many pieces and leave one CTA to read
// them all back.
//
// One CTA = one (weight tile, token tile, K split), warp specialised (192 threads):
//   warp 0      TMA producer: W[128 x 64] and X[BN x 64] tiles (128-byte swizzle) into a
//               STAGES-deep ring. The split sizes keep a CTA's whole K slice within the ring, so
//               all of its loads are in flight at once; the weight tiles of the first STAGES
//               stages are issued before griddepcontrol.wait (weights do not depend on the
//               previous kernel), the activation tiles after it.
//   warp 1      allocates TMEM and issues tcgen05.mma (one elected thread).
//   warps 2..5  epilogue: tcgen05.ld the accumulator into an fp32 partial tile in the drained
//               ring. After a cluster barrier every rank sums one slice of the tile over all
//               ranks' shared memory (distributed shared memory loads, rank order, so the sum is
//               deterministic) and stores it; a second barrier keeps each partial alive until
//               its peers have read it.
// Rings of at most ~110 KB let two CTAs share an SM for token tiles up to 128 rows.
#pragma once

namespace cl {

constexpr int THREADS_CL = 192;
constexpr int kMaxClusterSplits = 8;  // portable cluster size

constexpr int ctas_per_sm_for(int bn) { return bn <= 128 ? 2 : 1; }
// Ring stages: ~110 KB so two CTAs share an SM (token tiles up to 128), ~220 KB otherwise. `wide`
// is the one-CTA-per-SM ring (up to 12 stages in 200 KB) for problems whose tiles cannot fill two
// CTAs per SM even at the largest cluster (o_proj and down_proj at decode widths: 16 tiles x 8
// splits = 128 CTAs); there the deeper ring keeps a CTA's whole K slice in flight.
constexpr int stages_for(int bn, bool wide = false) {
  const int stage = BM * BK * 2 + bn * BK * 2;
  const int budget = (wide ? 200 : bn <= 128 ? 110 : 220) * 1024;
  const int cap = wide ? 12 : 8;
  return budget / stage < cap ? budget / stage : cap;
}

template <int BN, int STAGES>
struct CCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = (uint32_t)pow2_at_least(BN);
  static constexpr uint32_t IDESC = Cfg<BN>::IDESC;
  static_assert(BN * BM * 4 <= STAGES * STAGE_BYTES, "fp32 partial tile must fit in the stage ring");
  static_assert(2 * STAGES * 8 + 3 * 8 + 4 <= BAR_BYTES, "barriers");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct CParams {
  __nv_bfloat16* c;
  int64_t ldc;
  int M, N, K;
  int splits, kb_per_split, num_kb;  // splits == cluster size along z
  int vec_store;                     // c 8-byte aligned and ldc % 4 == 0
  int32_t* status;
  float* parts;                      // EPI 3: fp32 partial planes, split z at parts + z * part_stride ([M][N])
  int64_t part_stride;
};

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(THREADS_CL, 1)
    gemm_cluster_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                        CParams p) {
  using C = CCfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  float* red = reinterpret_cast<float*>(smem);  // [BN][BM] fp32 partial tile, after the main loop
  cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int wtile = blockIdx.x, mtile = blockIdx.y, split = blockIdx.z;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, p.num_kb);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  if (warp != 0) pdl_wait();  // the producer waits after issuing the weight tiles

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&map_w);
      prefetch_tensormap(&map_x);
      const int npre = min(STAGES, kb1 - kb0);
      for (int i = 0; i < npre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
        tma_load_2d(smem + i * C::STAGE_BYTES, &map_w, &full[i], (kb0 + i) * BK, wtile * BM);
      }
      pdl_wait();
      for (int i = 0; i < npre; ++i)
        tma_load_2d(smem + i * C::STAGE_BYTES + C::A_BYTES, &map_x, &full[i], (kb0 + i) * BK, mtile * BN);
      int stage = npre % STAGES;
      uint32_t phase = (npre == STAGES) ? 1u : 0u;
      int issued = npre;
      for (int kb = kb0 + npre; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) break;
        uint8_t* a = smem + stage * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
        tma_load_2d(a, &map_w, &full[stage], kb * BK, wtile * BM);
        tma_load_2d(a + C::A_BYTES, &map_x, &full[stage], kb * BK, mtile * BN);
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // Load j lands in stage j % STAGES and completes that barrier's phase of parity
      // (j / STAGES) & 1: wait (bounded) for the last load of every stage, so no copy is still in
      // flight when the ring is reused for the partial tile or the CTA exits.
      for (int j = max(0, issued - STAGES); j < issued; ++j)
        mbar_wait(&full[j % STAGES], (uint32_t)((j / STAGES) & 1), p.status);
    }
    __syncwarp();  // the warp reaches the block and cluster barriers converged
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, p.status)) break;
        tc_fence_after();
        const uint32_t a = smem_u32(smem + stage * C::STAGE_BYTES);
        const uint32_t b = a + C::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_bf16(tmem, sw128_desc(a + kk * 32), sw128_desc(b + kk * 32), C::IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      umma_commit(accum);
    }
    __syncwarp();
  }
  // the producer's loads have all landed and the MMA warp has issued its final commit
  __syncthreads();
  if constexpr (EPI == 3) {
    // Unreduced: this split's fp32 partial goes straight to its plane (a warp stores 128
    // consecutive bytes of one token row per instruction); the consumer sums the planes.
    if (warp >= 2) {
      const int q = warp & 3;
      const bool ok = mbar_wait(accum, 0, p.status);
      tc_fence_after();
      const int n = wtile * BM + q * 32 + lane;
      float* plane = p.parts + (int64_t)split * p.part_stride;
      if (ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = mtile * BN + c0 + j;
            if (c0 + j < BN && m < p.M && n < p.N) plane[(int64_t)m * p.N + n] = v[j];
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, C::TMEM_COLS);
    }
    return;
  }
  if (warp >= 2) {
    // TMEM -> this CTA's fp32 partial tile red[token][weight row] in the stage ring, free once the
    // accumulator barrier fires (every MMA, the ring's only reader, has completed)
    const int q = warp & 3;
    const bool ok = mbar_wait(accum, 0, p.status);
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < BN) red[(c0 + j) * BM + q * 32 + lane] = v[j];
      }
    }
  }
  tc_fence_before();
  // Every thread of every CTA of the cluster passes both cluster barriers exactly once, error
  // paths included, so no CTA can wait on one that has left.
  cluster.sync();
  {
    // Rank r sums slice r of the tile over all ranks in rank order and stores it as bf16 (4
    // consecutive weight rows = 4 consecutive output columns of one token per element).
    const int ns = p.splits;
    const int rank = (int)cluster.block_rank();
    constexpr int kVec = BM / 4;  // float4 per token row of the partial tile
    constexpr int kTotal = BN * kVec;
    const int per = (kTotal + ns - 1) / ns;
    const int e_beg = rank * per;
    const int e_end = min(e_beg + per, kTotal);
    const int m_base = mtile * BN;
    const float4* src[kMaxClusterSplits];
#pragma unroll
    for (int sp = 0; sp < kMaxClusterSplits; ++sp)
      src[sp] = ns == 1 ? reinterpret_cast<const float4*>(red)
                        : cluster.map_shared_rank(reinterpret_cast<const float4*>(red), sp < ns ? sp : 0);
    constexpr int U = 4;  // elements in flight per thread
    for (int e0 = e_beg + (int)threadIdx.x; e0 < e_end; e0 += U * THREADS_CL) {
      float4 acc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int e = e0 + u * THREADS_CL;
        acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e < e_end) {
          acc[u] = src[0][e];
#pragma unroll
          for (int sp = 1; sp < kMaxClusterSplits; ++sp)
            if (sp < ns) {
              const float4 t = src[sp][e];
              acc[u].x += t.x;
              acc[u].y += t.y;
              acc[u].z += t.z;
              acc[u].w += t.w;
            }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int e = e0 + u * THREADS_CL;
        if (e >= e_end) continue;
        const int gm = m_base + e / kVec;
        const int gn = wtile * BM + (e % kVec) * 4;
        if (gm >= p.M || gn >= p.N) continue;
        if constexpr (EPI == 1) {
          // (gate_j, up_j, gate_j+1, up_j+1) -> act[j], act[j+1], j = gn / 2 (N % 4 == 0 here)
          const float g0 = round_bf16(acc[u].x), u0 = round_bf16(acc[u].y);
          const float g1 = round_bf16(acc[u].z), u1 = round_bf16(acc[u].w);
          const float s0 = round_bf16(g0 / (1.f + expf(-g0)));
          const float s1 = round_bf16(g1 / (1.f + expf(-g1)));
          __nv_bfloat16* dst = p.c + (int64_t)gm * p.ldc + gn / 2;
          dst[0] = f_to_bf16(s0 * u0);
          dst[1] = f_to_bf16(s1 * u1);
        } else {
          __nv_bfloat16* dst = p.c + (int64_t)gm * p.ldc + gn;
          if (p.vec_store && gn + 3 < p.N) {
            *reinterpret_cast<uint2*>(dst) =
                make_uint2(pack_bf16x2(acc[u].x, acc[u].y), pack_bf16x2(acc[u].z, acc[u].w));
          } else {
            const float a4[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
            for (int j = 0; j < 4 && gn + j < p.N; ++j) dst[j] = f_to_bf16(a4[j]);
          }
        }
      }
    }
  }
  cluster.sync();  // peers finished reading this CTA's partial tile
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side of the split mode
template <int BN, int STAGES>
static cudaLaunchConfig_t cluster_config(const void* kernel, dim3 grid, int splits, cudaStream_t st,
                                         cudaLaunchAttribute (&attr)[2]) {
  (void)kernel;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(THREADS_CL);
  cfg.dynamicSmemBytes = CCfg<BN, STAGES>::SMEM;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = splits;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cfg;
}

// Split s <= want with the least estimated time. A launch of `clusters` clusters of s CTAs (one per
// output tile) runs in ceil(clusters / max_active(s)) waves (cudaOccupancyMaxActiveClusters,
// queried once per size), and each CTA does 1/s of the tile's K work: time ~ waves / s. Ties go to
// fewer waves (less fixed cost per wave).
template <int BN, int STAGES, int EPI>
static int schedulable_splits(int want, int clusters) {
  static std::mutex mu;
  static int max_active[kMaxClusterSplits + 1];
  static bool known[kMaxClusterSplits + 1] = {};
  std::lock_guard<std::mutex> lock(mu);
  int best = 1, best_waves = 0;
  double best_cost = 0.0;
  for (int s = 1; s <= want; ++s) {
    if (!known[s]) {
      cudaLaunchAttribute attr[2];
      cudaLaunchConfig_t cfg = cluster_config<BN, STAGES>(nullptr, dim3(1, 1, s), s, nullptr, attr);
      int n = 0;
      max_active[s] =
          cudaOccupancyMaxActiveClusters(&n, gemm_cluster_kernel<BN, STAGES, EPI>, &cfg) == cudaSuccess ? n : 0;
      cudaGetLastError();
      known[s] = true;
    }
    if (max_active[s] <= 0) continue;
    const int waves = (clusters + max_active[s] - 1) / max_active[s];
    const double cost = (double)waves / s;
    if (best_waves == 0 || cost < best_cost - 1e-9 || (cost < best_cost + 1e-9 && waves < best_waves)) {
      best = s;
      best_waves = waves;
      best_cost = cost;
    }
  }
  return best;
}

template <int BN, int STAGES, int EPI>
static int launch_cluster_with(const CUtensorMap& mw, const CUtensorMap& mx, CParams p, int tiles_n, int tiles_m,
                               int slots, cudaStream_t st) {
  using C = CCfg<BN, STAGES>;
  static int attr_state = 0;
  if (attr_state == 0) {
    attr_state = cudaFuncSetAttribute(gemm_cluster_kernel<BN, STAGES, EPI>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) == cudaSuccess ? 1 : -1;
    prefer_max_shared(reinterpret_cast<const void*>(gemm_cluster_kernel<BN, STAGES, EPI>));
  }
  if (attr_state != 1) return CDB_ERR_CUDA;
  // Fill the resident CTA slots with (weight tile, token tile, K split) CTAs, at least two
  // k-blocks per split.
  const int tiles = tiles_n * tiles_m;
  int want = tiles >= slots ? 1 : slots / tiles;
  want = min(want, max(1, p.num_kb / 2));
  want = max(1, min(want, kMaxClusterSplits));
  int s = schedulable_splits<BN, STAGES, EPI>(want, tiles);
  int kb_per = (p.num_kb + s - 1) / s;
  s = (p.num_kb + kb_per - 1) / kb_per;  // no empty split
  p.splits = s;
  p.kb_per_split = kb_per;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg =
      cluster_config<BN, STAGES>(nullptr, dim3(tiles_n, tiles_m, s), s, st, attr);
  return cudaLaunchKernelEx(&cfg, gemm_cluster_kernel<BN, STAGES, EPI>, mw, mx, p) == cudaSuccess ? CDB_OK
                                                                                                 : CDB_ERR_CUDA;
}

// Two CTAs per SM with ~110 KB rings, or, when even the largest clusters leave SMs without a
// second CTA (tiles x 8 <= SMs), one CTA per SM with the wide ring. In a 24-GEMM graph at 80
// tokens the wide ring took o_proj 2048x2048 from 8.3 to 7.8 us and down 2048x5632 from 11.8 to
// 10.9 us, and was slower for QKV (48 tiles) and gate/up (88 tiles), which fill two CTAs per SM.
template <int BN, int EPI>
static int launch_cluster(const CUtensorMap& mw, const CUtensorMap& mx, CParams p, int tiles_n, int tiles_m,
                          int num_sms, cudaStream_t st) {
  if constexpr (BN <= 128) {
    if (tiles_n * tiles_m * kMaxClusterSplits <= num_sms)
      return launch_cluster_with<BN, stages_for(BN, true), EPI>(mw, mx, p, tiles_n, tiles_m, num_sms, st);
  }
  return launch_cluster_with<BN, stages_for(BN), EPI>(mw, mx, p, tiles_n, tiles_m, num_sms * ctas_per_sm_for(BN), st);
}

// Split count of the unreduced mode: fill the resident CTA slots, at least two k-blocks per
// split, at most kPartSplitsPreferred planes (every plane is written by the GEMM and read back by
// the consumer; in a graph of 24 o_proj + norm pairs at 80 rows, 4-6 planes took 9.1-9.3 us per
// pair against 10.4 us at 16 and 11.1 us for the reduced GEMM + norm). Callers may pass up to
// kMaxPartSplits.
constexpr int kMaxPartSplits = 16;
constexpr int kPartSplitsPreferred = 6;
static int partial_splits(int bn, int tiles, int num_kb, int num_sms) {
  const int slots = num_sms * (bn <= 128 ? 2 : 1);
  int want = tiles >= slots ? 1 : slots / tiles;
  want = min(want, max(1, num_kb / 2));
  want = max(1, min(want, kPartSplitsPreferred));
  const int kb_per = (num_kb + want - 1) / want;
  return (num_kb + kb_per - 1) / kb_per;  // no empty split
}

template <int BN>
static int launch_partials(const CUtensorMap& mw, const CUtensorMap& mx, CParams p, int tiles_n, int tiles_m,
                           cudaStream_t st) {
  constexpr int STAGES = stages_for(BN);
  using C = CCfg<BN, STAGES>;
  static int attr_state = 0;
  if (attr_state == 0) {
    attr_state = cudaFuncSetAttribute(gemm_cluster_kernel<BN, STAGES, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      C::SMEM) == cudaSuccess ? 1 : -1;
    prefer_max_shared(reinterpret_cast<const void*>(gemm_cluster_kernel<BN, STAGES, 3>));
  }
  if (attr_state != 1) return CDB_ERR_CUDA;
  const int s = p.splits;
  p.kb_per_split = (p.num_kb + s - 1) / s;
  if ((p.num_kb + p.kb_per_split - 1) / p.kb_per_split != s) return CDB_ERR_INVALID_ARGUMENT;  // an empty split
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles_n, tiles_m, s);
  cfg.blockDim = dim3(THREADS_CL);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_cluster_kernel<BN, STAGES, 3>, mw, mx, p) == cudaSuccess ? CDB_OK
                                                                                               : CDB_ERR_CUDA;
}

}  // namespace cl
