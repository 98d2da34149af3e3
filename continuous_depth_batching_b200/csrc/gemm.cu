// bf16 tensor-core GEMM for sm_100a on tcgen05/TMEM: C[M,N] = X[M,K] * W[N,K]^T.
//
// Decode-shaped problems have few token rows (M <= 256) and wide weights (N up to 49152), so
// the weight is the MMA "A" operand (128 weight rows per tile, UMMA M=128) and the token rows
// are the MMA "B" operand (UMMA N = BN in {32,64,128,256}); the fp32 accumulator lives in
// tensor memory as [128 lanes = weight rows] x [BN columns = token rows].
//
// One CTA = one (weight tile, token tile, K split), warp specialised:
//   warp 0      TMA producer: 2-D tile loads of W[128 x 64] and X[BN x 64] (128-byte swizzle)
//               into a STAGES-deep ring, completion on "full" mbarriers;
//   warp 1      allocates TMEM and issues tcgen05.mma (one elected thread), releasing each
//               stage with tcgen05.commit onto its "empty" mbarrier;
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each warp reads its 32-lane quarter)
//               into an fp32 tile in the drained stage ring.
// Split-K (for the projections whose weight tiles cannot fill 148 SMs otherwise) keeps the
// splits of one tile in one thread-block cluster (grid z = cluster z = splits <= 8): after a
// cluster barrier every CTA reduces one slice of the tile from all ranks' shared memory
// (distributed shared memory loads, rank order, so the sum is deterministic) and stores it as
// bf16 with 8-byte vector stores. No global partials, counters or second pass.
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
constexpr int THREADS = 192;
constexpr int kMaxClusterSplits = 8;  // portable cluster size

// Token-tile widths of at most 128 run two CTAs per SM (stage ring within ~110 KB), wider ones one
// (ring within ~220 KB); the ring depth follows from the stage size, capped at 8.
constexpr int ctas_per_sm_for(int bn) { return bn <= 128 ? 2 : 1; }
constexpr int stages_for(int bn) {
  const int stage = BM * BK * 2 + bn * BK * 2;
  const int budget = (bn <= 128 ? 110 : 220) * 1024;
  return budget / stage < 8 ? budget / stage : 8;
}

template <int BN, int STAGES>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  // tcgen05.alloc takes a power of two >= 32 columns
  static constexpr uint32_t TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  // kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, M=128, N=BN.
  static constexpr uint32_t IDESC =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
  static_assert(BN * BM * 4 <= STAGES * STAGE_BYTES, "fp32 partial tile must fit in the stage ring");
};

struct Params {
  __nv_bfloat16* c;
  int64_t ldc;
  int M, N, K;
  int splits, kb_per_split, num_kb;  // splits == cluster size along z
  int vec_store;                     // c 8-byte aligned and ldc % 4 == 0
  int32_t* status;
  // EPI 2 (LM head + argmax): per-token running keys, completion counter, outputs
  unsigned long long* keys;
  int32_t* done;
  int total_ctas;
  int64_t* out_ids;
  const int32_t* out_rows;
  const int32_t* token_rows;
  int32_t* token_table;
};

// Orderable 64-bit key of (bf16 logit v, vocab index n): larger v wins, then the smaller index
// (torch.argmax returns the first maximum).
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

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
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
}

// EPI 0: store c[m, n] = bf16(acc). EPI 1 (SwiGLU): weight rows are gate/up pairs
// (row 2j = gate_j, row 2j+1 = up_j) and c[m, j] = bf16(bf16(silu(bf16(g))) * bf16(u)), the
// rounding of OuroMLP's act_fn(gate_proj(x)) * up_proj(x) in bf16. EPI 2 (LM head + greedy
// argmax, unsplit): no logits are stored; each token's argmax over the bf16 logits of the tile's
// vocab rows is folded into keys[m] with atomicMax, and the last CTA writes the token ids.
template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, Params p) {
  using C = Cfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  float* red = reinterpret_cast<float*>(smem);  // [BN][BM] fp32 partial tile, after the mainloop
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
  if (warp != 0) pdl_wait();  // the producer waits after prefetching weights

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&map_w);
      prefetch_tensormap(&map_x);
      // Weights do not depend on the previous kernel: fill the first stages' weight tiles
      // before waiting on it, then add the activation tiles.
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
      // (j / STAGES) & 1. Wait (bounded) for the last load of every stage, so that no copy is
      // still in flight when the ring is reused for the partial tile or the CTA exits.
      for (int j = max(0, issued - STAGES); j < issued; ++j)
        mbar_wait(&full[j % STAGES], (uint32_t)((j / STAGES) & 1), p.status);
    }
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
        for (int kk = 0; kk < BK / 16; ++kk) {
          umma_bf16(tmem, sw128_desc(a + kk * 32), sw128_desc(b + kk * 32), C::IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
        }
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
  // The producer's loads have all landed and the MMA warp has issued its final commit.
  __syncthreads();
  if (warp >= 2) {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    // TMEM -> this CTA's fp32 partial tile red[token][weight row] in the stage ring, which is
    // free once the accumulator barrier fires (every MMA, the ring's only reader, completed).
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool ok = mbar_wait(accum, 0, p.status);
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, r);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < BN) red[(c0 + j) * BM + q * 32 + lane] = __uint_as_float(r[j]);
      }
    }
  }
  tc_fence_before();
  // Every thread of every CTA of the cluster passes both cluster barriers exactly once, error
  // paths included, so no CTA can wait on one that has left.
  cluster.sync();

  if constexpr (EPI == 2) {
    // One warp per token: the max over this tile's 128 vocab rows, then one atomic per token.
    __shared__ int s_last;
    const int m_base = mtile * BN;
    for (int m = warp; m < BN && m_base + m < p.M; m += THREADS / 32) {
      const float4 v = reinterpret_cast<const float4*>(red)[m * (BM / 4) + lane];
      const float vals[4] = {v.x, v.y, v.z, v.w};
      unsigned long long best = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = wtile * BM + lane * 4 + j;
        if (n < p.N) {
          const unsigned long long k = argmax_key(round_bf16(vals[j]), n);
          best = k > best ? k : best;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
      }
      if (lane == 0 && best != 0) atomicMax(p.keys + m_base + m, best);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      s_last = atomicAdd(p.done, 1) == p.total_ctas - 1;
    }
    __syncthreads();
    if (s_last) {
      // every other CTA's atomics precede its counter increment: read and reset the keys
      __threadfence();
      for (int m = threadIdx.x; m < p.M; m += THREADS) {
        const unsigned long long k = atomicExch(p.keys + m, 0ull);
        const int64_t id = (int64_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        const int orow = p.out_rows ? p.out_rows[m] : m;
        if (orow >= 0) p.out_ids[orow] = id;
        if (p.token_rows != nullptr && p.token_rows[m] >= 0) p.token_table[p.token_rows[m]] = (int32_t)id;
      }
      if (threadIdx.x == 0) atomicExch(p.done, 0);
    }
  } else
  // Deterministic K-split reduction through distributed shared memory: the cluster holds the
  // tile's `splits` CTAs; rank r sums slice r of the tile over all ranks in rank order and
  // stores it as bf16 (4 consecutive weight rows = 4 consecutive output columns per thread).
  {
    const int ns = p.splits;
    const int rank = (int)cluster.block_rank();
    constexpr int kVec = BM / 4;  // float4 per token row of the partial tile
    constexpr int kTotal = BN * kVec;
    const int per = (kTotal + ns - 1) / ns;
    const int e_beg = rank * per;
    const int e_end = min(e_beg + per, kTotal);
    const int m_base = mtile * BN;
    const bool vec_store = p.vec_store;
    // Element e of the tile is float4 e of every rank's partial (token e / kVec, weight rows
    // 4 * (e % kVec) ..). Without a split the partial is this CTA's own shared memory.
    const float4* src[kMaxClusterSplits];
#pragma unroll
    for (int sp = 0; sp < kMaxClusterSplits; ++sp)
      src[sp] = ns == 1 ? reinterpret_cast<const float4*>(red)
                        : cluster.map_shared_rank(reinterpret_cast<const float4*>(red), sp < ns ? sp : 0);
    constexpr int U = 4;  // elements in flight per thread
    for (int e0 = e_beg + (int)threadIdx.x; e0 < e_end; e0 += U * THREADS) {
      float4 acc[U];
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int e = e0 + q * THREADS;
        if (e < e_end) {
          acc[q] = src[0][e];
#pragma unroll
          for (int sp = 1; sp < kMaxClusterSplits; ++sp)
            if (sp < ns) {
              const float4 t = src[sp][e];
              acc[q].x += t.x;
              acc[q].y += t.y;
              acc[q].z += t.z;
              acc[q].w += t.w;
            }
        }
      }
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int e = e0 + q * THREADS;
        if (e >= e_end) continue;
        const int gm = m_base + e / kVec;
        const int gn = wtile * BM + (e % kVec) * 4;
        if (gm >= p.M || gn >= p.N) continue;
        if constexpr (EPI == 1) {
          // N % 4 == 0 here: (gate_j, up_j, gate_j+1, up_j+1) -> act[j], act[j+1], j = gn / 2.
          const float g0 = round_bf16(acc[q].x), u0 = round_bf16(acc[q].y);
          const float g1 = round_bf16(acc[q].z), u1 = round_bf16(acc[q].w);
          const float s0 = round_bf16(g0 / (1.f + expf(-g0)));
          const float s1 = round_bf16(g1 / (1.f + expf(-g1)));
          *reinterpret_cast<uint32_t*>(p.c + (int64_t)gm * p.ldc + gn / 2) = pack_bf16x2(s0 * u0, s1 * u1);
        } else {
          __nv_bfloat16* dst = p.c + (int64_t)gm * p.ldc + gn;
          if (vec_store && gn + 3 < p.N) {
            *reinterpret_cast<uint2*>(dst) =
                make_uint2(pack_bf16x2(acc[q].x, acc[q].y), pack_bf16x2(acc[q].z, acc[q].w));
          } else {
            const float a4[4] = {acc[q].x, acc[q].y, acc[q].z, acc[q].w};
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

template <int BN, int STAGES>
static cudaLaunchConfig_t launch_config(dim3 grid, int splits, cudaStream_t st, cudaLaunchAttribute (&attr)[2]) {
  using C = Cfg<BN, STAGES>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
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

// Split s <= want with the least estimated time. A launch of `clusters` clusters of s CTAs (one
// cluster per output tile) runs in ceil(clusters / max_active(s)) waves, max_active from
// cudaOccupancyMaxActiveClusters (queried once per size and remembered), and each CTA does 1/s of
// the tile's K work: time ~ waves / s. Ties go to fewer waves (less fixed cost per wave).
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
      cudaLaunchConfig_t cfg = launch_config<BN, STAGES>(dim3(1, 1, s), s, nullptr, attr);
      int n = 0;
      max_active[s] = cudaOccupancyMaxActiveClusters(&n, gemm_kernel<BN, STAGES, EPI>, &cfg) == cudaSuccess ? n : 0;
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
static int launch(const CUtensorMap& mw, const CUtensorMap& mx, Params p, int tiles_n, int tiles_m, int splits,
                  cudaStream_t st) {
  using C = Cfg<BN, STAGES>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(gemm_kernel<BN, STAGES, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return CDB_ERR_CUDA;
    attr_set = true;
  }
  prefer_max_shared(reinterpret_cast<const void*>(gemm_kernel<BN, STAGES, EPI>));
  int s = schedulable_splits<BN, STAGES, EPI>(splits, tiles_n * tiles_m);
  int kb_per = (p.num_kb + s - 1) / s;
  s = (p.num_kb + kb_per - 1) / kb_per;  // no empty split
  p.splits = s;
  p.kb_per_split = kb_per;
  p.total_ctas = tiles_n * tiles_m * s;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = launch_config<BN, STAGES>(dim3(tiles_n, tiles_m, s), s, st, attr);
  return cudaLaunchKernelEx(&cfg, gemm_kernel<BN, STAGES, EPI>, mw, mx, p) == cudaSuccess ? CDB_OK : CDB_ERR_CUDA;
}

// Token-tile width for M token rows: M rounded up to a multiple of 16 (the UMMA N step for
// M = 128) up to 256; wider problems tile the tokens by 256.
static int tile_n_for(int M) { return M >= 256 ? 256 : ((max(M, 16) + 15) / 16) * 16; }
static int ctas_per_sm(int bn) { return ctas_per_sm_for(bn); }

}  // namespace gemm
}  // namespace cdb

using namespace cdb;

namespace cdb {
namespace gemm {

// Shared host path of the plain and SwiGLU GEMMs: c = epilogue(x[M,K] * w[N,K]^T).
template <int EPI>
static int run(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int M, int N, int K,
               int splits, int num_sms, int32_t* status, cudaStream_t st, const Params* epi2 = nullptr) {
  if (K % 8 != 0 || ldx % 8 != 0 || ldw % 8 != 0 || ldx < K || ldw < K) return CDB_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) return CDB_ERR_INVALID_ARGUMENT;
  const int bn = tile_n_for(M);
  const int tiles_n = (N + BM - 1) / BM;
  const int tiles_m = (M + bn - 1) / bn;
  const int num_kb = (K + BK - 1) / BK;
  if (num_sms <= 0) num_sms = 148;
  int s = splits;
  if (s <= 0) {
    // Fill the resident CTA slots with (weight tile, token tile, K split) CTAs, at least two
    // k-blocks per split.
    const int tiles = tiles_n * tiles_m;
    const int slots = num_sms * ctas_per_sm(bn);
    s = tiles >= slots ? 1 : slots / tiles;
    s = min(s, max(1, num_kb / 2));
  }
  s = max(1, min(min(s, kMaxClusterSplits), num_kb));
  if (EPI == 2) s = 1;  // the argmax epilogue reads whole (unsplit) logit tiles
  CUtensorMap mw, mx;
  int rc = matrix_map(&mw, w, N, K, ldw, BM);
  if (rc != CDB_OK) return rc;
  rc = matrix_map(&mx, x, M, K, ldx, bn);
  if (rc != CDB_OK) return rc;
  Params p;
  p.c = static_cast<__nv_bfloat16*>(c);
  p.ldc = ldc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.splits = s;
  p.kb_per_split = num_kb;
  p.num_kb = num_kb;
  p.vec_store = ((reinterpret_cast<uintptr_t>(c) & 7) == 0 && ldc % 4 == 0) ? 1 : 0;
  p.status = status;
  p.keys = epi2 ? epi2->keys : nullptr;
  p.done = epi2 ? epi2->done : nullptr;
  p.total_ctas = 0;
  p.out_ids = epi2 ? epi2->out_ids : nullptr;
  p.out_rows = epi2 ? epi2->out_rows : nullptr;
  p.token_rows = epi2 ? epi2->token_rows : nullptr;
  p.token_table = epi2 ? epi2->token_table : nullptr;
  switch (bn) {
    case 16:
      return launch<16, stages_for(16), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 32:
      return launch<32, stages_for(32), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 48:
      return launch<48, stages_for(48), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 64:
      return launch<64, stages_for(64), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 80:
      return launch<80, stages_for(80), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 96:
      return launch<96, stages_for(96), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 112:
      return launch<112, stages_for(112), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 128:
      return launch<128, stages_for(128), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 144:
      return launch<144, stages_for(144), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 160:
      return launch<160, stages_for(160), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 176:
      return launch<176, stages_for(176), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 192:
      return launch<192, stages_for(192), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 208:
      return launch<208, stages_for(208), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 224:
      return launch<224, stages_for(224), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 240:
      return launch<240, stages_for(240), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    case 256:
      return launch<256, stages_for(256), EPI>(mw, mx, p, tiles_n, tiles_m, s, st);
    default:
      return CDB_ERR_UNSUPPORTED;
  }
}

}  // namespace gemm
}  // namespace cdb

extern "C" int cdb_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* c, int64_t ldc, int M,
                             int N, int K, int splits, float* workspace, int64_t workspace_elems, int32_t* counters,
                             int num_counters, int num_sms, int32_t* status, void* stream) {
  (void)workspace;
  (void)workspace_elems;
  (void)counters;
  (void)num_counters;
  if (M <= 0 || N <= 0 || K <= 0) return M == 0 ? CDB_OK : CDB_ERR_INVALID_ARGUMENT;
  if (ldc < N) return CDB_ERR_INVALID_ARGUMENT;
  return cdb::gemm::run<0>(x, ldx, w, ldw, c, ldc, M, N, K, splits, num_sms, status, static_cast<cudaStream_t>(stream));
}

extern "C" int cdb_mlp_gateup_silu_gemm(const void* x, int64_t ldx, const void* w_gate_up, int64_t ldw, void* act,
                                        int64_t ld_act, int M, int inter, int K, int splits, int num_sms,
                                        int32_t* status, void* stream) {
  if (M <= 0 || inter <= 0 || K <= 0) return M == 0 ? CDB_OK : CDB_ERR_INVALID_ARGUMENT;
  if (inter % 2 != 0 || ld_act < inter || ld_act % 2 != 0 || (reinterpret_cast<uintptr_t>(act) & 3))
    return CDB_ERR_INVALID_ARGUMENT;
  return cdb::gemm::run<1>(x, ldx, w_gate_up, ldw, act, ld_act, M, 2 * inter, K, splits, num_sms, status,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int cdb_lm_head_argmax(const void* x, int64_t ldx, const void* w, int64_t ldw, int M, int vocab, int K,
                                  int64_t* out_ids, const int32_t* out_rows, const int32_t* token_rows,
                                  int32_t* token_table, uint64_t* keys, int32_t* done, int num_sms,
                                  int32_t* status, void* stream) {
  if (M <= 0 || vocab <= 0 || K <= 0) return M == 0 ? CDB_OK : CDB_ERR_INVALID_ARGUMENT;
  if (out_ids == nullptr || keys == nullptr || done == nullptr || (token_rows != nullptr && token_table == nullptr))
    return CDB_ERR_INVALID_ARGUMENT;
  cdb::gemm::Params e;
  e.keys = reinterpret_cast<unsigned long long*>(keys);
  e.done = done;
  e.out_ids = out_ids;
  e.out_rows = out_rows;
  e.token_rows = token_rows;
  e.token_table = token_table;
  return cdb::gemm::run<2>(x, ldx, w, ldw, nullptr, 0, M, vocab, K, 1, num_sms, status,
                           static_cast<cudaStream_t>(stream), &e);
}

extern "C" int64_t cdb_gemm_workspace_elems(int M, int N, int K, int num_sms) {
  (void)M;
  (void)N;
  (void)K;
  (void)num_sms;
  return 0;  // K splits reduce inside a thread-block cluster; no global workspace
}
