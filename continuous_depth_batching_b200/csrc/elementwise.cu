// Row-wise fused kernels of the CDB recurrent step: the sandwich RMSNorms (with the
// residual add, the exit-gate dot product and the hidden-bank scatter fused in), SwiGLU,
// greedy argmax, the prelude embedding gather, device block-table edits, the last_exited
// KV copy and the cumulative-hazard exit decision.
//
// All math is fp32; results are rounded to bf16 exactly where the reference's PyTorch bf16
// ops round (each elementwise op stores a bf16 tensor), so outputs match it up to the
// summation order of the row reductions.
#include <type_traits>

#include "cdb_common.cuh"

namespace cdb {

constexpr int kRowThreads = 256;
constexpr int kMaxChunks = 6;  // rows up to 256 threads x 6 x 8 = 12288 elements

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

// A bf16 row held as NC 8-element chunks per thread (chunk c of thread t covers elements
// (c * kRowThreads + t) * 8 ..). NC is the smallest count that covers the row, so registers
// scale with the row width.
template <int NC>
struct RowRegs {
  float v[NC][8];
};

template <int NC>
struct RowRaw {
  uint4 w[NC];
};

// Raw 16-byte chunks of a bf16 row (zeros past `hidden`); issued early, converted later.
template <int NC>
__device__ __forceinline__ void load_raw(const __nv_bfloat16* row, int hidden, RowRaw<NC>& r) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int d = (c * kRowThreads + threadIdx.x) * 8;
    r.w[c] = d < hidden ? *reinterpret_cast<const uint4*>(row + d) : make_uint4(0u, 0u, 0u, 0u);
  }
}

template <int NC>
__device__ __forceinline__ void unpack_row(const RowRaw<NC>& w, RowRegs<NC>& r) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    r.v[c][0] = bf16lo(w.w[c].x);
    r.v[c][1] = bf16hi(w.w[c].x);
    r.v[c][2] = bf16lo(w.w[c].y);
    r.v[c][3] = bf16hi(w.w[c].y);
    r.v[c][4] = bf16lo(w.w[c].z);
    r.v[c][5] = bf16hi(w.w[c].z);
    r.v[c][6] = bf16lo(w.w[c].w);
    r.v[c][7] = bf16hi(w.w[c].w);
  }
}

template <int NC>
__device__ __forceinline__ void load_row(const __nv_bfloat16* row, int hidden, RowRegs<NC>& r) {
  RowRaw<NC> w;
  load_raw(row, hidden, w);
  unpack_row(w, r);
}

template <int NC>
__device__ __forceinline__ void store_row(__nv_bfloat16* row, int hidden, const RowRegs<NC>& r) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int d = (c * kRowThreads + threadIdx.x) * 8;
    if (d < hidden) {
      uint4 w;
      w.x = pack_bf16x2(r.v[c][0], r.v[c][1]);
      w.y = pack_bf16x2(r.v[c][2], r.v[c][3]);
      w.z = pack_bf16x2(r.v[c][4], r.v[c][5]);
      w.w = pack_bf16x2(r.v[c][6], r.v[c][7]);
      *reinterpret_cast<uint4*>(row + d) = w;
    }
  }
}

// In-register OuroRMSNorm with preloaded weights: r <- weight * bf16(r * rsqrt(mean(r^2) + eps)),
// all rounded to bf16.
template <int NC>
__device__ __forceinline__ void rms_inplace(RowRegs<NC>& r, const RowRaw<NC>& weight, int hidden, float eps,
                                            float* red) {
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int k = 0; k < 8; ++k) ss = fmaf(r.v[c][k], r.v[c][k], ss);
  const float var = block_sum(ss, red) / (float)hidden;
  const float inv = rsqrtf(var + eps);
  RowRegs<NC> g;
  unpack_row(weight, g);
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int k = 0; k < 8; ++k) r.v[c][k] = round_bf16(g.v[c][k] * round_bf16(r.v[c][k] * inv));
}

// Norm kernels load their weights before pdl_wait() (weights never depend on the preceding
// kernel) and issue every row load before the first reduction, so a launch costs one memory
// round trip after its predecessor finishes instead of one per operand.
template <int NC>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_kernel(const __nv_bfloat16* x, int64_t xs, const int32_t* x_rows,
                                                              const __nv_bfloat16* w, __nv_bfloat16* y, int64_t ys,
                                                              __nv_bfloat16* xc, int64_t xcs, int hidden, float eps) {
  pdl_trigger();
  RowRaw<NC> wr;
  load_raw(w, hidden, wr);
  pdl_wait();
  __shared__ float red[32];
  const int r = blockIdx.x;
  const int src = x_rows ? x_rows[r] : r;
  if (src < 0) return;
  RowRegs<NC> v;
  load_row(x + (int64_t)src * xs, hidden, v);
  if (xc) store_row(xc + (int64_t)r * xcs, hidden, v);
  rms_inplace(v, wr, hidden, eps, red);
  store_row(y + (int64_t)r * ys, hidden, v);
}

// Row of a = bf16(sum over the split-K partial planes, in plane order) from fp32 partials
// ap[z * pstride + d] (the GEMM's own reduction order, so a equals what the GEMM would store).
template <int NC>
__device__ __forceinline__ void load_parts(const float* ap, int nparts, int64_t pstride, int hidden, RowRegs<NC>& r) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int d = (c * kRowThreads + threadIdx.x) * 8;
    float s[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) s[k] = 0.f;
    if (d < hidden) {
      const float4* p0 = reinterpret_cast<const float4*>(ap + d);
      float4 lo = p0[0], hi = p0[1];
      s[0] = lo.x, s[1] = lo.y, s[2] = lo.z, s[3] = lo.w, s[4] = hi.x, s[5] = hi.y, s[6] = hi.z, s[7] = hi.w;
#pragma unroll 4
      for (int z = 1; z < nparts; ++z) {
        const float4* pz = reinterpret_cast<const float4*>(ap + z * pstride + d);
        lo = pz[0];
        hi = pz[1];
        s[0] += lo.x, s[1] += lo.y, s[2] += lo.z, s[3] += lo.w, s[4] += hi.x, s[5] += hi.y, s[6] += hi.z, s[7] += hi.w;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) r.v[c][k] = round_bf16(s[k]);
  }
}

// a is either a bf16 row (a, as) or, when ap != nullptr, the sum of nparts fp32 split-K partial
// planes ap + z * pstride (row r at ap + r * hidden) that a split GEMM left unreduced.
template <int NC>
__global__ void __launch_bounds__(kRowThreads) add_rmsnorm_kernel(__nv_bfloat16* x, int64_t xs, const __nv_bfloat16* a,
                                                                  int64_t as, const float* ap, int nparts,
                                                                  int64_t pstride, const __nv_bfloat16* wa,
                                                                  const __nv_bfloat16* wn, __nv_bfloat16* y, int64_t ys,
                                                                  const int32_t* y_rows, const __nv_bfloat16* gw,
                                                                  const __nv_bfloat16* gb, __nv_bfloat16* gout,
                                                                  int hidden, float eps) {
  pdl_trigger();
  RowRaw<NC> war, wnr, gwr;
  load_raw(wa, hidden, war);
  load_raw(wn, hidden, wnr);
  if (gw) load_raw(gw, hidden, gwr);
  pdl_wait();
  __shared__ float red[32];
  const int r = blockIdx.x;
  const int dst = y_rows ? y_rows[r] : r;
  if (dst < 0) return;
  RowRaw<NC> ar, xr;
  RowRegs<NC> av, xv;
  load_raw(x + (int64_t)r * xs, hidden, xr);
  if (ap != nullptr) {
    load_parts(ap + (int64_t)r * hidden, nparts, pstride, hidden, av);
  } else {
    load_raw(a + (int64_t)r * as, hidden, ar);
    unpack_row(ar, av);
  }
  rms_inplace(av, war, hidden, eps, red);
  unpack_row(xr, xv);
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int k = 0; k < 8; ++k) xv.v[c][k] = round_bf16(xv.v[c][k] + av.v[c][k]);
  store_row(x + (int64_t)r * xs, hidden, xv);
  rms_inplace(xv, wnr, hidden, eps, red);
  store_row(y + (int64_t)dst * ys, hidden, xv);
  if (gw) {
    RowRegs<NC> g;
    unpack_row(gwr, g);
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int k = 0; k < 8; ++k) dot = fmaf(g.v[c][k], xv.v[c][k], dot);
    dot = block_sum(dot, red);
    if (threadIdx.x == 0) gout[r] = f_to_bf16(dot + bf16_to_f(gb[0]));
  }
}

__global__ void silu_mul_kernel(const __nv_bfloat16* gu, int64_t gs, __nv_bfloat16* act, int64_t as, int inter) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.y;
  const int d = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (d >= inter) return;
  const uint4 g = *reinterpret_cast<const uint4*>(gu + (int64_t)r * gs + d);
  const uint4 u = *reinterpret_cast<const uint4*>(gu + (int64_t)r * gs + inter + d);
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
  const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
  uint32_t ow[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float g0 = bf16lo(gw[k]), g1 = bf16hi(gw[k]);
    const float s0 = round_bf16(g0 / (1.f + expf(-g0)));
    const float s1 = round_bf16(g1 / (1.f + expf(-g1)));
    ow[k] = pack_bf16x2(s0 * bf16lo(uw[k]), s1 * bf16hi(uw[k]));
  }
  *reinterpret_cast<uint4*>(act + (int64_t)r * as + d) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

__device__ __forceinline__ void better(float v, int i, float& bv, int& bi) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

__global__ void __launch_bounds__(512) argmax_kernel(const __nv_bfloat16* logits, int64_t stride, int vocab,
                                                     int64_t* out, const int32_t* out_rows, const int32_t* token_rows,
                                                     int32_t* token_table) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int r = blockIdx.x;
  const __nv_bfloat16* row = logits + (int64_t)r * stride;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  if ((vocab & 7) == 0 && (stride & 7) == 0) {
    for (int d = threadIdx.x * 8; d < vocab; d += blockDim.x * 8) {
      const uint4 w = *reinterpret_cast<const uint4*>(row + d);
      better(bf16lo(w.x), d, bv, bi);
      better(bf16hi(w.x), d + 1, bv, bi);
      better(bf16lo(w.y), d + 2, bv, bi);
      better(bf16hi(w.y), d + 3, bv, bi);
      better(bf16lo(w.z), d + 4, bv, bi);
      better(bf16hi(w.z), d + 5, bv, bi);
      better(bf16lo(w.w), d + 6, bv, bi);
      better(bf16hi(w.w), d + 7, bv, bi);
    }
  } else {
    for (int d = threadIdx.x; d < vocab; d += blockDim.x) better(bf16_to_f(row[d]), d, bv, bi);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(ov, oi, bv, bi);
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    bv = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      better(ov, oi, bv, bi);
    }
    if (lane == 0) {
      if (bi == 0x7fffffff) bi = 0;
      const int orow = out_rows ? out_rows[r] : r;
      if (orow >= 0) out[orow] = bi;
      if (token_rows != nullptr && token_rows[r] >= 0) token_table[token_rows[r]] = bi;
    }
  }
}

__global__ void embed_kernel(const __nv_bfloat16* table, int hidden, int vocab, const int32_t* ids,
                             const int32_t* id_src, const int32_t* token_table, __nv_bfloat16* out, int64_t os,
                             const int32_t* out_rows, float scale, int32_t* status) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  const int dst = out_rows ? out_rows[r] : r;
  if (dst < 0) return;
  int id = ids ? ids[r] : -1;
  if (id < 0 && id_src != nullptr) {
    const int slot = id_src[r];
    id = slot >= 0 ? token_table[slot] : -1;  // a negative slot has no device token: reported below
  }
  __nv_bfloat16* o = out + (int64_t)dst * os;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_error(status, CDB_ERR_INDEX);
    for (int d = threadIdx.x; d < hidden; d += blockDim.x) o[d] = f_to_bf16(0.f);
    return;
  }
  const __nv_bfloat16* src = table + (int64_t)id * hidden;
  if (scale != 1.f) {
    // wte(ids) * scale in bf16: fp32 product rounded once (modeling_huginn.py:431)
    for (int d = threadIdx.x; d < hidden; d += blockDim.x) o[d] = f_to_bf16(bf16_to_f(src[d]) * scale);
  } else if ((hidden & 7) == 0) {
    for (int d = threadIdx.x * 8; d < hidden; d += blockDim.x * 8)
      *reinterpret_cast<uint4*>(o + d) = *reinterpret_cast<const uint4*>(src + d);
  } else {
    for (int d = threadIdx.x; d < hidden; d += blockDim.x) o[d] = src[d];
  }
}

// Huginn's sandwich-norm row step, general enough for every block boundary and stage edge:
//   v = xs[x_rows ? x_rows[r] : r]; if a: v = bf16(v + a[r]); if w1: v = rmsnorm(v; w1);
//   if xd: xd[xd_rows ? xd_rows[r] : r] = v (skipped when that index < 0);
//   if w2: y[r] = rmsnorm(v; w2).
// (HuginnBlock.forward modeling_huginn.py:333-336: x = norm_2(attn + x), norm_3(x); x = norm_4(mlp
// + x), then the next block's norm_1; run_coda :454-460: ln_f before and after the coda blocks.)
template <int NC>
__global__ void __launch_bounds__(kRowThreads) sandwich_norm_kernel(
    const __nv_bfloat16* xs, int64_t xss, const int32_t* x_rows, const __nv_bfloat16* a, int64_t as,
    const __nv_bfloat16* w1, __nv_bfloat16* xd, int64_t xds, const int32_t* xd_rows, const __nv_bfloat16* w2,
    __nv_bfloat16* y, int64_t ys, int hidden, float eps) {
  pdl_trigger();
  RowRaw<NC> w1r, w2r;
  if (w1) load_raw(w1, hidden, w1r);
  if (w2) load_raw(w2, hidden, w2r);
  pdl_wait();
  __shared__ float red[32];
  const int r = blockIdx.x;
  const int src = x_rows ? x_rows[r] : r;
  if (src < 0) return;
  RowRaw<NC> xr, ar;
  load_raw(xs + (int64_t)src * xss, hidden, xr);
  if (a) load_raw(a + (int64_t)r * as, hidden, ar);
  RowRegs<NC> v;
  unpack_row(xr, v);
  if (a) {
    RowRegs<NC> av;
    unpack_row(ar, av);
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int k = 0; k < 8; ++k) v.v[c][k] = round_bf16(av.v[c][k] + v.v[c][k]);
  }
  if (w1) rms_inplace(v, w1r, hidden, eps, red);
  if (xd) {
    const int dst = xd_rows ? xd_rows[r] : r;
    if (dst >= 0) store_row(xd + (int64_t)dst * xds, hidden, v);
  }
  if (w2) {
    rms_inplace(v, w2r, hidden, eps, red);
    store_row(y + (int64_t)r * ys, hidden, v);
  }
}

// latent_diff (models/huginn/exit_gates.py:33-40) in bf16 tensors, as the adapter computes it:
// d = bf16(new - old); out[r] = bf16(bf16(||d||) / max(bf16(||new||), 1e-9)), norms accumulated
// in fp32. new row rows[r] (r when rows == NULL), old row r; rows[r] < 0 skips row r.
template <int NC>
__global__ void __launch_bounds__(kRowThreads) latent_diff_kernel(const __nv_bfloat16* nw, int64_t ns,
                                                                  const __nv_bfloat16* old, int64_t os,
                                                                  const int32_t* rows, int hidden,
                                                                  __nv_bfloat16* out) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int r = blockIdx.x;
  const int nr = rows ? rows[r] : r;
  if (nr < 0) return;
  RowRegs<NC> a, b;
  load_row(nw + (int64_t)nr * ns, hidden, a);
  load_row(old + (int64_t)r * os, hidden, b);
  float sd = 0.f, sn = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float d = round_bf16(a.v[c][k] - b.v[c][k]);
      sd = fmaf(d, d, sd);
      sn = fmaf(a.v[c][k], a.v[c][k], sn);
    }
  sd = block_sum(sd, red);
  sn = block_sum(sn, red);
  if (threadIdx.x == 0) {
    const float nd = round_bf16(sqrtf(sd));
    const float nn = fmaxf(round_bf16(sqrtf(sn)), 1e-9f);
    out[r] = f_to_bf16(nd / nn);
  }
}

// dst[r] = src[rows[r]] for bf16 rows of `hidden` elements (rows[r] < 0: row r is zeroed).
__global__ void gather_rows_kernel(const __nv_bfloat16* src, int64_t ss, const int32_t* rows, int hidden,
                                   __nv_bfloat16* dst, int64_t ds) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  const int sr = rows[r];
  __nv_bfloat16* o = dst + (int64_t)r * ds;
  if (sr < 0) {
    for (int d = threadIdx.x; d < hidden; d += blockDim.x) o[d] = f_to_bf16(0.f);
    return;
  }
  const __nv_bfloat16* x = src + (int64_t)sr * ss;
  if ((hidden & 7) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(o)) & 15) == 0) {
    for (int d = threadIdx.x * 8; d < hidden; d += blockDim.x * 8)
      *reinterpret_cast<uint4*>(o + d) = *reinterpret_cast<const uint4*>(x + d);
  } else {
    for (int d = threadIdx.x; d < hidden; d += blockDim.x) o[d] = x[d];
  }
}

__global__ void block_table_update_kernel(int32_t* table, int64_t stride, const int32_t* edits, int n) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  table[(int64_t)edits[3 * i] * stride + edits[3 * i + 1]] = edits[3 * i + 2];
}

__global__ void exit_kv_copy_kernel(__nv_bfloat16* kv, int64_t kv_rows, int64_t row_elems, const int32_t* rows,
                                    const int32_t* src_layers, const int32_t* dst_layers) {
  pdl_trigger();
  pdl_wait();
  const int64_t row = rows[blockIdx.x];
  const int pair = blockIdx.y;
  const int src = src_layers[pair], dst = dst_layers[pair];
  for (int kvsel = 0; kvsel < 2; ++kvsel) {
    const uint4* s = reinterpret_cast<const uint4*>(kv + ((int64_t)(2 * src + kvsel) * kv_rows + row) * row_elems);
    uint4* d = reinterpret_cast<uint4*>(kv + ((int64_t)(2 * dst + kvsel) * kv_rows + row) * row_elems);
    for (int i = threadIdx.x; i < row_elems / 8; i += blockDim.x) d[i] = s[i];
  }
}

__global__ void exit_hazard_kernel(const void* signal, int signal_bf16, const int32_t* slots, const int32_t* steps,
                                   const int8_t* reset, double* cdf, double* surv, int8_t* exit_out, int n,
                                   int min_steps, double threshold) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const int s = slots[r];
  if (s < 0) {
    exit_out[r] = 0;
    return;
  }
  if (reset != nullptr && reset[r]) {
    cdf[s] = 0.0;
    surv[s] = 1.0;
  }
  float h;
  if (signal_bf16) {
    const float x = bf16_to_f(static_cast<const __nv_bfloat16*>(signal)[r]);
    h = round_bf16(1.f / (1.f + expf(-x)));
  } else {
    const float x = static_cast<const float*>(signal)[r];
    h = 1.f / (1.f + expf(-x));
  }
  const double hd = (double)h;
  const double c = cdf[s] + hd * surv[s];
  cdf[s] = c;
  surv[s] = surv[s] * (1.0 - hd);
  exit_out[r] = (steps[r] + 1 >= min_steps && c >= threshold) ? 1 : 0;
}

static inline int check_launch() { return cudaPeekAtLastError() == cudaSuccess ? CDB_OK : CDB_ERR_CUDA; }

}  // namespace cdb

using namespace cdb;

extern "C" int cdb_version(void) { return 100; }

extern "C" const char* cdb_status_string(int status) {
  switch (status) {
    case CDB_OK:
      return "ok";
    case CDB_ERR_INVALID_ARGUMENT:
      return "invalid argument";
    case CDB_ERR_UNSUPPORTED:
      return "unsupported shape";
    case CDB_ERR_CUDA:
      return "CUDA launch error";
    case CDB_ERR_DEVICE_TIMEOUT:
      return "device-side wait ran out of iterations";
    case CDB_ERR_TMA_ENCODE:
      return "TMA tensor map encoding failed";
    case CDB_ERR_INDEX:
      return "device-side index out of range";
    case CDB_ERR_SCRATCH_LIMIT:
      return "call exceeds the static scratch limits (head_dim <= 128, num_heads <= 128, plan <= 32768 units)";
    default:
      return "unknown status";
  }
}

// Calls f(std::integral_constant<int, NC>) with NC = the chunks per thread covering `hidden`.
template <typename F>
static void with_row_chunks(int hidden, F&& f) {
  switch (max(1, (hidden + kRowThreads * 8 - 1) / (kRowThreads * 8))) {
    case 1: f(std::integral_constant<int, 1>{}); break;
    case 2: f(std::integral_constant<int, 2>{}); break;
    case 3: f(std::integral_constant<int, 3>{}); break;
    case 4: f(std::integral_constant<int, 4>{}); break;
    case 5: f(std::integral_constant<int, 5>{}); break;
    default: f(std::integral_constant<int, kMaxChunks>{}); break;
  }
}

extern "C" int cdb_rmsnorm(const void* x, int64_t x_stride, const int32_t* x_rows, const void* weight, void* y,
                           int64_t y_stride, void* x_copy, int64_t x_copy_stride, int num_rows, int hidden, float eps,
                           void* stream) {
  if (hidden % 8 != 0 || hidden > kRowThreads * kMaxChunks * 8 || num_rows < 0) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  with_row_chunks(hidden, [&](auto nc) {
    launch_pdl(rmsnorm_kernel<decltype(nc)::value>, dim3(num_rows), dim3(kRowThreads), 0,
               static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x), x_stride, x_rows,
               static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(y), y_stride,
               static_cast<__nv_bfloat16*>(x_copy), x_copy_stride, hidden, eps);
  });
  return check_launch();
}

extern "C" int cdb_add_rmsnorm(void* x, int64_t x_stride, const void* a, int64_t a_stride, const void* w_a,
                               const void* w_next, void* y, int64_t y_stride, const int32_t* y_rows,
                               const void* gate_w, const void* gate_b, void* gate_out, int num_rows, int hidden,
                               float eps, void* stream) {
  if (hidden % 8 != 0 || hidden > kRowThreads * kMaxChunks * 8 || num_rows < 0) return CDB_ERR_INVALID_ARGUMENT;
  if (gate_w != nullptr && (gate_b == nullptr || gate_out == nullptr)) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  with_row_chunks(hidden, [&](auto nc) {
    launch_pdl(add_rmsnorm_kernel<decltype(nc)::value>, dim3(num_rows), dim3(kRowThreads), 0,
               static_cast<cudaStream_t>(stream), static_cast<__nv_bfloat16*>(x), x_stride,
               static_cast<const __nv_bfloat16*>(a), a_stride, static_cast<const float*>(nullptr), 0, (int64_t)0,
               static_cast<const __nv_bfloat16*>(w_a),
               static_cast<const __nv_bfloat16*>(w_next), static_cast<__nv_bfloat16*>(y), y_stride, y_rows,
               static_cast<const __nv_bfloat16*>(gate_w), static_cast<const __nv_bfloat16*>(gate_b),
               static_cast<__nv_bfloat16*>(gate_out), hidden, eps);
  });
  return check_launch();
}

extern "C" int cdb_add_rmsnorm_parts(void* x, int64_t x_stride, const float* a_parts, int num_parts,
                                     int64_t part_stride, const void* w_a, const void* w_next, void* y,
                                     int64_t y_stride, const int32_t* y_rows, const void* gate_w, const void* gate_b,
                                     void* gate_out, int num_rows, int hidden, float eps, void* stream) {
  if (hidden % 8 != 0 || hidden > kRowThreads * kMaxChunks * 8 || num_rows < 0) return CDB_ERR_INVALID_ARGUMENT;
  if (gate_w != nullptr && (gate_b == nullptr || gate_out == nullptr)) return CDB_ERR_INVALID_ARGUMENT;
  if (a_parts == nullptr || num_parts < 1 || (reinterpret_cast<uintptr_t>(a_parts) & 15) || part_stride % 4 != 0 ||
      part_stride < (int64_t)num_rows * hidden)
    return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  with_row_chunks(hidden, [&](auto nc) {
    launch_pdl(add_rmsnorm_kernel<decltype(nc)::value>, dim3(num_rows), dim3(kRowThreads), 0,
               static_cast<cudaStream_t>(stream), static_cast<__nv_bfloat16*>(x), x_stride,
               static_cast<const __nv_bfloat16*>(nullptr), (int64_t)0, a_parts, num_parts, part_stride,
               static_cast<const __nv_bfloat16*>(w_a), static_cast<const __nv_bfloat16*>(w_next),
               static_cast<__nv_bfloat16*>(y), y_stride, y_rows, static_cast<const __nv_bfloat16*>(gate_w),
               static_cast<const __nv_bfloat16*>(gate_b), static_cast<__nv_bfloat16*>(gate_out), hidden, eps);
  });
  return check_launch();
}

extern "C" int cdb_silu_mul(const void* gu, int64_t gu_stride, void* act, int64_t act_stride, int num_rows, int inter,
                            void* stream) {
  if (inter % 8 != 0 || num_rows < 0) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  const int threads = 128;
  dim3 grid((inter / 8 + threads - 1) / threads, num_rows);
  launch_pdl(silu_mul_kernel, dim3(grid), dim3(threads), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(gu), gu_stride, static_cast<__nv_bfloat16*>(act), act_stride, inter);
  return check_launch();
}

extern "C" int cdb_gather_rows(const void* src, int64_t src_stride, const int32_t* rows, int num_rows, int hidden,
                               void* dst, int64_t dst_stride, void* stream) {
  if (hidden <= 0 || num_rows < 0 || rows == nullptr) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  launch_pdl(gather_rows_kernel, dim3(num_rows), dim3(128), 0, static_cast<cudaStream_t>(stream),
             static_cast<const __nv_bfloat16*>(src), src_stride, rows, hidden, static_cast<__nv_bfloat16*>(dst),
             dst_stride);
  return check_launch();
}

extern "C" int cdb_argmax(const void* logits, int64_t stride, int num_rows, int vocab, int64_t* out,
                          const int32_t* out_rows, const int32_t* token_rows, int32_t* token_table, void* stream) {
  if (vocab <= 0 || num_rows < 0 || (token_rows != nullptr && token_table == nullptr)) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  launch_pdl(argmax_kernel, dim3(num_rows), dim3(512), 0, static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(logits),
                                                                         stride, vocab, out, out_rows, token_rows, token_table);
  return check_launch();
}

extern "C" int cdb_embed(const void* table, int hidden, int vocab, const int32_t* ids, const int32_t* id_src,
                         const int32_t* token_table, void* out, int64_t out_stride, const int32_t* out_rows,
                         int num_rows, float scale, int32_t* status, void* stream) {
  if (hidden <= 0 || vocab <= 0 || num_rows < 0 || (ids == nullptr && id_src == nullptr)) return CDB_ERR_INVALID_ARGUMENT;
  if (id_src != nullptr && token_table == nullptr) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  launch_pdl(embed_kernel, dim3(num_rows), dim3(128), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(table), hidden, vocab, ids, id_src, token_table,
      static_cast<__nv_bfloat16*>(out), out_stride, out_rows, scale, status);
  return check_launch();
}

extern "C" int cdb_sandwich_norm(const void* x_src, int64_t x_src_stride, const int32_t* x_rows, const void* add,
                                 int64_t add_stride, const void* w1, void* x_dst, int64_t x_dst_stride,
                                 const int32_t* x_dst_rows, const void* w2, void* y, int64_t y_stride, int num_rows,
                                 int hidden, float eps, void* stream) {
  if (hidden % 8 != 0 || hidden > kRowThreads * kMaxChunks * 8 || num_rows < 0 || (w2 != nullptr && y == nullptr))
    return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  with_row_chunks(hidden, [&](auto nc) {
    launch_pdl(sandwich_norm_kernel<decltype(nc)::value>, dim3(num_rows), dim3(kRowThreads), 0,
               static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x_src), x_src_stride, x_rows,
               static_cast<const __nv_bfloat16*>(add), add_stride, static_cast<const __nv_bfloat16*>(w1),
               static_cast<__nv_bfloat16*>(x_dst), x_dst_stride, x_dst_rows, static_cast<const __nv_bfloat16*>(w2),
               static_cast<__nv_bfloat16*>(y), y_stride, hidden, eps);
  });
  return check_launch();
}

extern "C" int cdb_latent_diff(const void* new_state, int64_t new_stride, const void* old_state, int64_t old_stride,
                               const int32_t* rows, int num_rows, int hidden, void* out, void* stream) {
  if (hidden % 8 != 0 || hidden > kRowThreads * kMaxChunks * 8 || num_rows < 0) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  with_row_chunks(hidden, [&](auto nc) {
    launch_pdl(latent_diff_kernel<decltype(nc)::value>, dim3(num_rows), dim3(kRowThreads), 0,
               static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(new_state), new_stride,
               static_cast<const __nv_bfloat16*>(old_state), old_stride, rows, hidden,
               static_cast<__nv_bfloat16*>(out));
  });
  return check_launch();
}

extern "C" int cdb_block_table_update(int32_t* table, int64_t stride, const int32_t* edits, int num_edits,
                                      void* stream) {
  if (num_edits < 0) return CDB_ERR_INVALID_ARGUMENT;
  if (num_edits == 0) return CDB_OK;
  launch_pdl(block_table_update_kernel, dim3((num_edits + 255) / 256), dim3(256), 0, static_cast<cudaStream_t>(stream), table, stride,
                                                                                                   edits, num_edits);
  return check_launch();
}

extern "C" int cdb_exit_kv_copy(void* kv_base, int num_cache_layers, int64_t kv_rows, int num_kv_heads, int head_dim,
                                const int32_t* rows, int num_rows, const int32_t* src_layers,
                                const int32_t* dst_layers, int num_pairs, void* stream) {
  const int64_t row_elems = (int64_t)num_kv_heads * head_dim;
  if (row_elems % 8 != 0 || num_rows < 0 || num_pairs < 0 || num_cache_layers <= 0) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0 || num_pairs == 0) return CDB_OK;
  dim3 grid(num_rows, num_pairs);
  launch_pdl(exit_kv_copy_kernel, dim3(grid), dim3(128), 0, static_cast<cudaStream_t>(stream), 
      static_cast<__nv_bfloat16*>(kv_base), kv_rows, row_elems, rows, src_layers, dst_layers);
  return check_launch();
}

extern "C" int cdb_exit_hazard(const void* signal, int signal_bf16, const int32_t* slots, const int32_t* steps,
                               const int8_t* reset, double* cdf, double* surv, int8_t* exit_out, int num_rows,
                               int min_steps, double threshold, void* stream) {
  if (num_rows < 0) return CDB_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return CDB_OK;
  launch_pdl(exit_hazard_kernel, dim3((num_rows + 127) / 128), dim3(128), 0, static_cast<cudaStream_t>(stream), 
      signal, signal_bf16, slots, steps, reset, cdf, surv, exit_out, num_rows, min_steps, threshold);
  return check_launch();
}
