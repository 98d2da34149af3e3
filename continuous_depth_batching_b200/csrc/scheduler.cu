// Device-side scheduling primitives of the CDB decode step: exit-gate evaluation with routing and
// compaction of one recurrent launch, the FIFO KV block allocator, and the per-launch block-table
// / cu_seq_lens build. All are integer (or scalar) work on a few hundred rows, so each is one CTA
// of 1024 threads whose order-dependent parts (FIFO pops, stable compaction) are block-wide scans;
// the order they produce is the order the reference's host code produces.
#include "cdb_common.cuh"

namespace cdb {

constexpr int kSchedThreads = 1024;

// Exclusive scan of one int per thread over the block; `total` receives the sum.
__device__ __forceinline__ int sched_scan(int v, int* s_warp, int& total) {
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

// ------------------------------------------------------------------ exit gate + routing
// Row r of a recurrent launch: policy-state slot hidden[r] (< 0: padding, not routed), step[r],
// replay depth depth[r] (< 0 or depth == NULL: none), reset[r] (a new token: clear its state).
// Live decision of this step (ExitPolicy.should_exit, exit_policy.py:150-169):
//   policy 1, cumulative hazard: h = bf16(sigmoid(x)); cdf += h*surv; surv *= 1-h;
//             d = step+1 >= min_steps && cdf >= threshold
//   policy 2, direct threshold:  d = step+1 >= min_steps && x < threshold
// Routing (continuous_api.py:1090-1203, 1250-1280, 1671-1724):
//   synchronous: exit = step == max_steps-1 || (replay ? step >= depth : d)
//   delayed:     exit = step == max_steps-1 || (replay ? step >= depth+1 : pending == 1), and this
//                step's d becomes the slot's pending decision for the routing after its next launch.
// Survivors and exits are compacted in row order (survivors return to the queue head in order,
// exits join the coda queue in order).
__global__ void __launch_bounds__(kSchedThreads) exit_gate_route_kernel(
    const __nv_bfloat16* signal, int64_t signal_stride, const int32_t* hidden, const int32_t* step,
    const int32_t* depth, const int8_t* reset, double* cdf, double* surv, int8_t* pending, int n, int policy,
    int delayed, int min_steps, int max_steps, double threshold, int8_t* exit_flag, int32_t* survivors,
    int32_t* exits, int32_t* counts) {
  pdl_trigger();
  pdl_wait();
  __shared__ int s_warp[32];
  int base_s = 0, base_e = 0;
  for (int start = 0; start < n; start += kSchedThreads) {
    const int r = start + threadIdx.x;
    int ex = 0, sv = 0;
    if (r < n) {
      const int s = hidden[r];
      if (s >= 0) {
        if (reset != nullptr && reset[r]) {
          cdf[s] = 0.0;
          surv[s] = 1.0;
          if (pending != nullptr) pending[s] = -1;
        }
        const int st = step[r];
        const bool can_exit = st + 1 >= min_steps;
        int d = 0;
        if (policy == 1) {
          const float x = bf16_to_f(signal[(int64_t)r * signal_stride]);
          const double h = (double)round_bf16(1.f / (1.f + expf(-x)));
          const double c = cdf[s] + h * surv[s];
          cdf[s] = c;
          surv[s] = surv[s] * (1.0 - h);
          d = can_exit && c >= threshold;
        } else if (policy == 2) {
          const float x = bf16_to_f(signal[(int64_t)r * signal_stride]);
          d = can_exit && (double)x < threshold;
        }
        const int dep = depth != nullptr ? depth[r] : -1;
        const bool forced = st == max_steps - 1;
        if (delayed) {
          const int prev = pending[s];
          ex = forced || (dep >= 0 ? st >= dep + 1 : prev == 1);
          pending[s] = policy != 0 ? (int8_t)d : (int8_t)-1;
        } else {
          ex = forced || (dep >= 0 ? st >= dep : d);
        }
        sv = !ex;
        exit_flag[r] = (int8_t)ex;
      } else {
        exit_flag[r] = -1;
      }
    }
    int tot_s, tot_e;
    const int os = sched_scan(sv, s_warp, tot_s);
    const int oe = sched_scan(ex, s_warp, tot_e);
    if (sv) survivors[base_s + os] = r;
    if (ex) exits[base_e + oe] = r;
    base_s += tot_s;
    base_e += tot_e;
  }
  if (threadIdx.x == 0) {
    counts[0] = base_s;
    counts[1] = base_e;
  }
}

// ------------------------------------------------------------------ FIFO KV block allocator
// Device mirror of BlockManager (continuous_batching/cache_manager.py:33-91): a ring of free block
// ids popped at the head and appended at the tail, so ids come out in exactly the order the
// reference's deque hands them out. state = {head, free count, num_blocks, peak allocated}.
// row_len[slot] counts the blocks in block-table row `slot`.
__global__ void block_pool_init_kernel(int32_t* ring, int32_t* state, int32_t* row_len, int num_rows,
                                       int num_blocks) {
  pdl_trigger();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < num_blocks; i += gridDim.x * blockDim.x) ring[i] = i;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < num_rows; i += gridDim.x * blockDim.x) row_len[i] = 0;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    state[0] = 0;
    state[1] = num_blocks;
    state[2] = num_blocks;
    state[3] = 0;
  }
}

// Requests in order: request j takes counts[j] blocks from the head into row slots[j] (appended
// after the row's current blocks), unless fewer are free or the row would pass `width`; then
// granted[j] = 0 and it takes nothing, while later requests still try (get_free_blocks returns
// None for that request alone, cache_manager.py:72-81).
__global__ void __launch_bounds__(kSchedThreads) block_alloc_kernel(int32_t* ring, int32_t* state, int32_t* row_len,
                                                                     int32_t* table, int64_t table_stride, int width,
                                                                     const int32_t* slots, const int32_t* counts,
                                                                     int n, int32_t* granted) {
  pdl_trigger();
  pdl_wait();
  __shared__ int s_off[kSchedThreads], s_col[kSchedThreads], s_cnt[kSchedThreads];
  __shared__ int s_head0;
  const int nb = state[2];
  for (int start = 0; start < n; start += kSchedThreads) {
    const int m = min(kSchedThreads, n - start);
    if (threadIdx.x == 0) {
      // Grant decisions are sequential: each depends on what the earlier requests took.
      const int head0 = state[0];
      int avail = state[1];
      int taken = 0;
      for (int k = 0; k < m; ++k) {
        const int j = start + k;
        const int slot = slots[j], cnt = counts[j];
        const int len = row_len[slot];
        const bool ok = cnt >= 0 && cnt <= avail && len + cnt <= width;
        granted[j] = ok ? 1 : 0;
        s_off[k] = taken;
        s_col[k] = len;
        s_cnt[k] = ok ? cnt : 0;
        if (ok) {
          taken += cnt;
          avail -= cnt;
          row_len[slot] = len + cnt;
        }
      }
      s_head0 = head0;
      state[0] = nb > 0 ? (head0 + taken) % nb : 0;
      state[1] = avail;
      if (nb - avail > state[3]) state[3] = nb - avail;
    }
    __syncthreads();
    for (int k = threadIdx.x; k < m; k += blockDim.x) {
      int32_t* row = table + (int64_t)slots[start + k] * table_stride;
      for (int b = 0; b < s_cnt[k]; ++b) row[s_col[k] + b] = ring[(s_head0 + s_off[k] + b) % nb];
    }
    __syncthreads();
  }
}

// Rows slots[j], in the order given: their blocks (columns 0 .. row_len-1, in column order) are
// appended at the ring's tail, the row is cleared to -1 and its length to 0 (a finished request's
// block list released in order, BlockManager.free_blocks). A slot may appear at most once.
__global__ void __launch_bounds__(kSchedThreads) block_free_kernel(int32_t* ring, int32_t* state, int32_t* row_len,
                                                                    int32_t* table, int64_t table_stride,
                                                                    const int32_t* slots, int n) {
  pdl_trigger();
  pdl_wait();
  __shared__ int s_warp[32];
  __shared__ int s_tail0;
  const int nb = state[2];
  for (int start = 0; start < n; start += kSchedThreads) {
    const int j = start + threadIdx.x;
    const int len = j < n ? row_len[slots[j]] : 0;
    int total;
    const int off = sched_scan(len, s_warp, total);
    if (threadIdx.x == 0) s_tail0 = nb > 0 ? (state[0] + state[1]) % nb : 0;
    __syncthreads();
    if (j < n) {
      int32_t* row = table + (int64_t)slots[j] * table_stride;
      for (int b = 0; b < len; ++b) {
        ring[(s_tail0 + off + b) % nb] = row[b];
        row[b] = -1;
      }
      row_len[slots[j]] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) state[1] += total;
    __syncthreads();
  }
}

// ------------------------------------------------------------------ per-launch tables
// The metadata a paged decode launch hands FlashAttention's kvcache branch
// (_prepare_recurrent_stage_buffers, model_runner.py:704-754): for rows i < n, block_table row i is
// the full block row of slot item_slot[i] (-1 past its blocks) and cu_seq_lens_k[i+1] =
// cu_seq_lens_k[i] + item_pos[i] + 1; cu_seq_lens_q = 0, 1, .., n. Padding rows n <= i < bucket
// get an all -1 row and plateaued cumsums. A row whose position is beyond its blocks sets
// CDB_ERR_INDEX (the reference raises ValueError).
__global__ void __launch_bounds__(kSchedThreads) build_tables_kernel(
    const int32_t* table, int64_t table_stride, const int32_t* row_len, int width, int block_size,
    const int32_t* item_slot, const int32_t* item_pos, int n, int bucket, int32_t* out, int64_t out_stride,
    int32_t* cu_q, int32_t* cu_k, int32_t* status) {
  pdl_trigger();
  pdl_wait();
  __shared__ int s_warp[32];
  int carry = 0;
  for (int start = 0; start < bucket; start += kSchedThreads) {
    const int i = start + threadIdx.x;
    int len_k = 0;
    if (i < n) {
      const int slot = item_slot[i], pos = item_pos[i];
      const int blocks = row_len[slot];
      len_k = pos + 1;
      if (pos < 0 || (int64_t)(pos + 1) > (int64_t)blocks * block_size) set_error(status, CDB_ERR_INDEX);
      const int32_t* src = table + (int64_t)slot * table_stride;
      for (int c = 0; c < width; ++c) out[(int64_t)i * out_stride + c] = c < blocks ? src[c] : -1;
    } else if (i < bucket) {
      for (int c = 0; c < width; ++c) out[(int64_t)i * out_stride + c] = -1;
    }
    int total;
    const int excl = sched_scan(len_k, s_warp, total);
    if (i < bucket) {
      cu_k[i + 1] = carry + excl + len_k;
      cu_q[i + 1] = min(i + 1, n);
    }
    carry += total;
  }
  if (threadIdx.x == 0) {
    cu_k[0] = 0;
    cu_q[0] = 0;
  }
}

}  // namespace cdb

using namespace cdb;

static inline int sched_launched() { return cudaPeekAtLastError() == cudaSuccess ? CDB_OK : CDB_ERR_CUDA; }

extern "C" int cdb_exit_gate_route(const void* signal, int64_t signal_stride, const int32_t* hidden,
                                   const int32_t* step, const int32_t* depth, const int8_t* reset, double* cdf,
                                   double* surv, int8_t* pending, int num_rows, int policy, int delayed,
                                   int min_steps, int max_steps, double threshold, int8_t* exit_flag,
                                   int32_t* survivors, int32_t* exits, int32_t* counts, void* stream) {
  if (num_rows < 0 || policy < 0 || policy > 2 || max_steps < 1 || hidden == nullptr || step == nullptr ||
      exit_flag == nullptr || survivors == nullptr || exits == nullptr || counts == nullptr)
    return CDB_ERR_INVALID_ARGUMENT;
  if (policy != 0 && (signal == nullptr || cdf == nullptr || surv == nullptr)) return CDB_ERR_INVALID_ARGUMENT;
  if (delayed && pending == nullptr) return CDB_ERR_INVALID_ARGUMENT;
  launch_pdl(exit_gate_route_kernel, dim3(1), dim3(kSchedThreads), 0, static_cast<cudaStream_t>(stream),
             static_cast<const __nv_bfloat16*>(signal), signal_stride, hidden, step, depth, reset, cdf, surv, pending,
             num_rows, policy, delayed, min_steps, max_steps, threshold, exit_flag, survivors, exits, counts);
  return sched_launched();
}

extern "C" int cdb_block_pool_init(int32_t* ring, int32_t* state, int32_t* row_len, int num_rows, int num_blocks,
                                   void* stream) {
  if (num_blocks < 0 || num_rows < 0 || ring == nullptr || state == nullptr || row_len == nullptr)
    return CDB_ERR_INVALID_ARGUMENT;
  const int items = num_blocks > num_rows ? num_blocks : num_rows;
  int blocks = (items + 255) / 256;
  blocks = blocks < 1 ? 1 : (blocks > 1184 ? 1184 : blocks);
  launch_pdl(block_pool_init_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream), ring, state,
             row_len, num_rows, num_blocks);
  return sched_launched();
}

extern "C" int cdb_block_alloc(int32_t* ring, int32_t* state, int32_t* row_len, int32_t* block_table,
                               int64_t block_table_stride, int width, const int32_t* slots, const int32_t* counts,
                               int num_requests, int32_t* granted, void* stream) {
  if (num_requests < 0 || width < 0 || block_table_stride < width || ring == nullptr || state == nullptr ||
      row_len == nullptr || block_table == nullptr || slots == nullptr || counts == nullptr || granted == nullptr)
    return CDB_ERR_INVALID_ARGUMENT;
  if (num_requests == 0) return CDB_OK;
  launch_pdl(block_alloc_kernel, dim3(1), dim3(kSchedThreads), 0, static_cast<cudaStream_t>(stream), ring, state,
             row_len, block_table, block_table_stride, width, slots, counts, num_requests, granted);
  return sched_launched();
}

extern "C" int cdb_block_free(int32_t* ring, int32_t* state, int32_t* row_len, int32_t* block_table,
                              int64_t block_table_stride, const int32_t* slots, int num_slots, void* stream) {
  if (num_slots < 0 || ring == nullptr || state == nullptr || row_len == nullptr || block_table == nullptr ||
      slots == nullptr)
    return CDB_ERR_INVALID_ARGUMENT;
  if (num_slots == 0) return CDB_OK;
  launch_pdl(block_free_kernel, dim3(1), dim3(kSchedThreads), 0, static_cast<cudaStream_t>(stream), ring, state,
             row_len, block_table, block_table_stride, slots, num_slots);
  return sched_launched();
}

extern "C" int cdb_build_tables(const int32_t* block_table, int64_t block_table_stride, const int32_t* row_len,
                                int width, int block_size, const int32_t* item_slot, const int32_t* item_pos,
                                int num_items, int bucket, int32_t* out_table, int64_t out_stride, int32_t* cu_seq_lens_q,
                                int32_t* cu_seq_lens_k, int32_t* status, void* stream) {
  if (num_items < 0 || bucket < num_items || width < 0 || block_size <= 0 || out_stride < width ||
      block_table == nullptr || row_len == nullptr || out_table == nullptr || cu_seq_lens_q == nullptr ||
      cu_seq_lens_k == nullptr || (num_items > 0 && (item_slot == nullptr || item_pos == nullptr)))
    return CDB_ERR_INVALID_ARGUMENT;
  launch_pdl(build_tables_kernel, dim3(1), dim3(kSchedThreads), 0, static_cast<cudaStream_t>(stream), block_table,
             block_table_stride, row_len, width, block_size, item_slot, item_pos, num_items, bucket, out_table,
             out_stride, cu_seq_lens_q, cu_seq_lens_k, status);
  return sched_launched();
}

// ------------------------------------------------------------------ scheduler tick on device queues
namespace cdb {

constexpr int kTickCap = 2048;  // items a queue may hold (both rings staged in shared memory)

// One CDBScheduler tick on device-resident queues (CDBScheduler.schedule_next, scheduler.py:101-140,
// with the queue operations of enqueue_depth / enqueue_depth_front / enqueue_coda, :142-186, and the
// slot-homogeneous FIFO pop of _schedule_recurrent_batch, :322-346), in the order the engine applies
// them between two launches: the last recurrent batch's survivors return to the head of the depth
// queue in batch order with their step advanced and its exits join the coda queue; prefill successors
// are appended; coda successors go to the head in order. Then the tick's work is chosen: a coda batch
// when the coda queue holds min_coda items, else prefill when the host admits it, else a recurrent
// batch of up to max_seqs items sharing the head item's KV slot (the others keep their order), else a
// coda flush. The rings are staged in shared memory and the order-dependent part runs on one thread:
// it is a few hundred integer steps.
__global__ void __launch_bounds__(kSchedThreads) schedule_tick_kernel(
    int32_t* state, int32_t* ready, int32_t* coda, int32_t* item_step, const int32_t* routed,
    const int8_t* exit_flag, int n_routed, const int32_t* back, int n_back, const int32_t* front, int n_front,
    int min_coda, int max_seqs, int prefill_admit, int slots, int32_t* out) {
  pdl_trigger();
  pdl_wait();
  __shared__ int32_t R[2][kTickCap], Q[2][kTickCap];
  __shared__ int s_rc, s_cc, s_kind, s_n, s_err;
  const int cap = state[4];
  const int rh = state[0], rc = state[1], ch = state[2], cc = state[3];
  if (cap <= 0 || cap > kTickCap || rc < 0 || rc > cap || cc < 0 || cc > cap || rh < 0 || ch < 0) {
    if (threadIdx.x == 0) {  // a ring the shared-memory staging cannot hold: report, change nothing
      out[0] = -1;
      out[1] = 0;
    }
    return;
  }
  for (int i = threadIdx.x; i < rc; i += blockDim.x) R[0][i] = ready[(rh + i) % cap];
  for (int i = threadIdx.x; i < cc; i += blockDim.x) Q[0][i] = coda[(ch + i) % cap];
  __syncthreads();
  if (threadIdx.x == 0) {
    int err = 0;
    int nr = rc, nc = cc, refills = state[5];
    int32_t* r = R[0];
    int32_t* rn = R[1];
    // survivors to the head in batch order (step + 1), exits to the coda queue
    int ns = 0;
    for (int i = 0; i < n_routed; ++i)
      if (!exit_flag[i]) ++ns;
    if (nr + ns + n_back + n_front > cap || nc + n_routed > cap) {
      err = 1;
    } else {
      int k = 0;
      for (int i = 0; i < n_routed; ++i) {
        const int id = routed[i];
        if (exit_flag[i]) {
          Q[0][nc++] = id;
        } else {
          item_step[id] += 1;
          rn[k++] = id;
        }
      }
      for (int i = 0; i < nr; ++i) rn[k++] = r[i];
      nr = k;
      int32_t* t = r;
      r = rn;
      rn = t;
      // prefill successors at the back (a step-0 item joining a non-empty queue is a refill)
      for (int i = 0; i < n_back; ++i) {
        if (item_step[back[i]] == 0 && nr > 0) ++refills;
        r[nr++] = back[i];
      }
      // coda successors to the head, in order (pushed one by one from the last)
      for (int i = n_front - 1; i >= 0; --i)
        if (item_step[front[i]] == 0 && nr + (n_front - 1 - i) > 0) ++refills;
      k = 0;
      for (int i = 0; i < n_front; ++i) rn[k++] = front[i];
      for (int i = 0; i < nr; ++i) rn[k++] = r[i];
      nr = k;
      t = r;
      r = rn;
      rn = t;
    }
    // the tick's work
    int kind = 0, n = 0;
    if (!err) {
      if (nc >= min_coda && nc > 0) {
        kind = 1;
      } else if (prefill_admit) {
        kind = 2;
      } else if (nr > 0) {
        kind = 3;
      } else if (nc > 0) {
        kind = 1;
      }
      if (kind == 1) {
        n = nc < max_seqs ? nc : max_seqs;
        for (int i = 0; i < n; ++i) out[2 + i] = Q[0][i];
        for (int i = n; i < nc; ++i) Q[0][i - n] = Q[0][i];
        nc -= n;
      } else if (kind == 3) {
        const int want = nr < max_seqs ? nr : max_seqs;
        const int target = min(item_step[r[0]], slots - 1);
        int d = 0, i = 0;
        for (; i < nr && n < want; ++i) {
          const int id = r[i];
          if (min(item_step[id], slots - 1) == target) {
            out[2 + n++] = id;
          } else {
            rn[d++] = id;
          }
        }
        for (; i < nr; ++i) rn[d++] = r[i];
        nr = d;
        r = rn;
      }
    }
    s_kind = kind;
    s_n = n;
    s_err = err;
    s_rc = nr;
    s_cc = nc;
    // publish the staged ready ring through buffer 0 for the parallel write-back
    if (!err && r != R[0])
      for (int i = 0; i < nr; ++i) R[0][i] = r[i];
    if (!err) state[5] = refills;
  }
  __syncthreads();
  const int nr = s_rc, nc = s_cc;
  if (!s_err) {  // on overflow the queues stay exactly as they were
    for (int i = threadIdx.x; i < nr; i += blockDim.x) ready[i] = R[0][i];
    for (int i = threadIdx.x; i < nc; i += blockDim.x) coda[i] = Q[0][i];
  }
  if (threadIdx.x == 0) {
    out[0] = s_err ? -1 : s_kind;
    out[1] = s_n;
    if (!s_err) {
      state[0] = 0;
      state[1] = nr;
      state[2] = 0;
      state[3] = nc;
    }
  }
}

}  // namespace cdb

extern "C" int cdb_schedule_tick(int32_t* queue_state, int32_t* ready, int32_t* coda, int32_t* item_step,
                                 const int32_t* routed, const int8_t* exit_flag, int num_routed, const int32_t* back,
                                 int num_back, const int32_t* front, int num_front, int min_coda_batch_size,
                                 int max_num_seqs, int prefill_admit, int kv_slots_per_layer, int32_t* out,
                                 void* stream) {
  if (queue_state == nullptr || ready == nullptr || coda == nullptr || item_step == nullptr || out == nullptr ||
      num_routed < 0 || num_back < 0 || num_front < 0 || min_coda_batch_size <= 0 || max_num_seqs <= 0 ||
      kv_slots_per_layer <= 0 || (num_routed > 0 && (routed == nullptr || exit_flag == nullptr)) ||
      (num_back > 0 && back == nullptr) || (num_front > 0 && front == nullptr))
    return CDB_ERR_INVALID_ARGUMENT;
  launch_pdl(schedule_tick_kernel, dim3(1), dim3(kSchedThreads), 0, static_cast<cudaStream_t>(stream), queue_state,
             ready, coda, item_step, routed, exit_flag, num_routed, back, num_back, front, num_front,
             min_coda_batch_size, max_num_seqs, prefill_admit, kv_slots_per_layer, out);
  return sched_launched();
}

extern "C" int cdb_schedule_queues_init(int32_t* queue_state, int capacity, void* stream) {
  if (queue_state == nullptr || capacity <= 0 || capacity > cdb::kTickCap) return CDB_ERR_INVALID_ARGUMENT;
  const int32_t init[8] = {0, 0, 0, 0, capacity, 0, 0, 0};
  return cudaMemcpyAsync(queue_state, init, sizeof(init), cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? CDB_OK
             : CDB_ERR_CUDA;
}
