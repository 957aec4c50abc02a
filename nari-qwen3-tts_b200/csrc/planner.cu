// GPU planner: page allocation and attention metadata for the next ragged
// batch, built on the device with no host round trip.
//
// State (one device buffer per page pool):
//   free bitmap u32[W]  (bit set = page free), W = ceil(total_pages / 32)
//   seq_len i32[slots], pos_start i32[slots], n_pages i32[slots]
//   page_table i32[slots * max_pages]
//
// Allocation reproduces the reference allocator exactly
// (executor/cache.py:135-184): rows are served in order and each takes the
// lowest free pages.  Row r needs missing_r pages; with M_r the exclusive
// prefix of missing over rows, row r receives the free pages of rank
// [M_r, M_r + missing_r) in ascending page order.  The rank -> page map is a
// popcount prefix over bitmap words plus a select inside one word, so every
// new page is found in parallel from one snapshot of the bitmap.
//
// Metadata reproduces PagedTalkerKV._metadata (executor/talker_kv.py:403-480):
// indptr over proposed page counts, proposed page lists, last_page_len =
// total % P or P, per-token write page/offset and position, padding rows on
// their private scratch page (last_page_len 1; prefill qo_len 0; decode
// writes slot 0 of it) and spare token slots spread over the scratch pages.
#include "common.cuh"

namespace nqt {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kMaxRows = 1024;
constexpr int kMaxWordsSmem = 16384;  // 524288 pages

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct StateView {
  uint32_t* bitmap;
  int32_t* seq_len;
  int32_t* pos_start;
  int32_t* n_pages;
  int32_t* table;
};

__host__ __device__ inline StateView state_view(void* base, int total_pages, int slots, int max_pages) {
  uint8_t* p = static_cast<uint8_t*>(base);
  const size_t words = (static_cast<size_t>(total_pages) + 31) / 32;
  StateView v;
  size_t off = 0;
  v.bitmap = reinterpret_cast<uint32_t*>(p + off);
  off = align256(off + 4 * words);
  v.seq_len = reinterpret_cast<int32_t*>(p + off);
  off = align256(off + 4 * static_cast<size_t>(slots));
  v.pos_start = reinterpret_cast<int32_t*>(p + off);
  off = align256(off + 4 * static_cast<size_t>(slots));
  v.n_pages = reinterpret_cast<int32_t*>(p + off);
  off = align256(off + 4 * static_cast<size_t>(slots));
  v.table = reinterpret_cast<int32_t*>(p + off);
  return v;
}

size_t state_bytes(int total_pages, int slots, int max_pages) {
  const size_t words = (static_cast<size_t>(total_pages) + 31) / 32;
  size_t off = align256(4 * words);
  off = align256(off + 4 * static_cast<size_t>(slots));
  off = align256(off + 4 * static_cast<size_t>(slots));
  off = align256(off + 4 * static_cast<size_t>(slots));
  off = align256(off + 4 * static_cast<size_t>(slots) * max_pages);
  return off;
}

// Exclusive block scan (kPlanThreads threads); returns the exclusive prefix
// and writes the block total to *total.
__device__ int block_excl_scan(int v, int* warp_buf, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) warp_buf[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_buf[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, w, o);
      if (lane >= o) w += y;
    }
    warp_buf[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int base = warp > 0 ? warp_buf[warp - 1] : 0;
  *total = warp_buf[31];
  return base + incl - v;
}

// Position of the n-th (0-based) set bit of m.
__device__ __forceinline__ int select_bit(uint32_t m, int n) {
  for (int i = 0; i < n; ++i) m &= m - 1;
  return __ffs(m) - 1;
}

struct PlanArgs {
  StateView st;
  int total_pages, slots, max_pages, page_size;
  const int32_t* row_slot;
  const int32_t* row_adv;
  int rows, token_capacity;
  const int32_t* scratch;
  int scratch_count, prefill;
  int32_t* qo_indptr;
  int32_t* kv_indptr;
  int32_t* kv_indices;
  int kv_capacity;
  int32_t* last_len;
  int64_t* positions;
  int64_t* write_pages;
  int64_t* write_offsets;
  int32_t* pending;
  int32_t* status;
};

__global__ void __launch_bounds__(kPlanThreads) plan_step_kernel(PlanArgs a) {
  extern __shared__ int32_t s_wpref[];  // [W + 1] free-page prefix over bitmap words
  __shared__ int s_warp[32];
  __shared__ int s_slot[kMaxRows], s_adv[kMaxRows], s_owned[kMaxRows], s_len[kMaxRows];
  __shared__ int s_mpref[kMaxRows + 1], s_kvpref[kMaxRows + 1], s_tpref[kMaxRows + 1];
  __shared__ int s_real[kMaxRows];
  __shared__ int s_fail, s_real_tokens;

  const int tid = threadIdx.x;
  const int P = a.page_size;
  const int W = (a.total_pages + 31) / 32;
  const int r = tid;
  const int pstride = a.max_pages + 1;

  // free pages per word and their prefix
  int carry = 0;
  for (int w0 = 0; w0 < W; w0 += kPlanThreads) {
    const int w = w0 + tid;
    const int c = w < W ? __popc(a.st.bitmap[w]) : 0;
    int tot;
    const int ex = block_excl_scan(c, s_warp, &tot);
    if (w < W) s_wpref[w] = carry + ex;
    carry += tot;
    __syncthreads();
  }
  if (tid == 0) s_wpref[W] = carry;
  const int free_count = carry;

  // per-row requirements
  int slot = -1, adv = 0, owned = 0, len = 0, need = 0;
  bool real = false;
  if (r < a.rows) {
    slot = a.row_slot[r];
    if (slot >= 0) {
      adv = a.row_adv[r];
      if (slot >= a.slots || adv < 1) {
        report(a.status, NQT_DEV_BAD_SLOT);
      } else {
        len = a.st.seq_len[slot];
        owned = a.st.n_pages[slot];
        need = (len + adv + P - 1) / P;
        if (need > a.max_pages || owned > need) {
          report(a.status, NQT_DEV_TABLE_FULL);
        } else {
          real = true;
        }
      }
    }
  }
  if (tid == 0) s_fail = 0;
  for (int attempt = 0; attempt < 2; ++attempt) {
    __syncthreads();
    if (s_fail) real = false;  // second pass: every row on scratch, nothing reserved
    const int missing = real ? need - owned : 0;
    const int kv_count = r < a.rows ? (real ? need : 1) : 0;
    const int ntok = r < a.rows ? (real ? adv : (a.prefill ? 0 : 1)) : 0;
    int tm, tkv, tt, treal;
    const int mp = block_excl_scan(missing, s_warp, &tm);
    const int kp = block_excl_scan(kv_count, s_warp, &tkv);
    const int tp = block_excl_scan(ntok, s_warp, &tt);
    block_excl_scan(real ? adv : 0, s_warp, &treal);
    if (r < a.rows) {
      s_mpref[r] = mp;
      s_kvpref[r] = kp;
      s_tpref[r] = tp;
      s_slot[r] = real ? slot : -1;
      s_adv[r] = real ? adv : 0;
      s_owned[r] = real ? owned : 0;
      s_len[r] = real ? len : 0;
      s_real[r] = real ? 1 : 0;
    }
    if (tid == 0) {
      s_mpref[a.rows] = tm;
      s_kvpref[a.rows] = tkv;
      s_tpref[a.rows] = tt;
      s_real_tokens = treal;
    }
    __syncthreads();
    if (attempt == 0) {
      if (tid == 0) {
        if (tm > free_count) {
          report(a.status, NQT_DEV_KV_EXHAUSTED);
          s_fail = 1;
        } else if (tkv > a.kv_capacity || (a.positions != nullptr && tt > a.token_capacity)) {
          report(a.status, NQT_DEV_CAPACITY);
          s_fail = 1;
        }
      }
      __syncthreads();
      if (!s_fail) break;
    }
  }

  // row-level metadata
  const int rows = a.rows;
  if (r < rows) {
    a.kv_indptr[r] = s_kvpref[r];
    const int total = s_len[r] + s_adv[r];
    a.last_len[r] = s_real[r] ? (total % P == 0 ? P : total % P) : 1;
    if (a.qo_indptr != nullptr) a.qo_indptr[r] = s_tpref[r];
    a.pending[r * pstride] = s_real[r] ? s_mpref[r + 1] - s_mpref[r] : -1;
  }
  if (tid == 0) {
    a.kv_indptr[rows] = s_kvpref[rows];
    if (a.qo_indptr != nullptr) a.qo_indptr[rows] = s_tpref[rows];
  }

  // new pages: rank q -> row (binary search) and page (word prefix + select)
  const int total_missing = s_mpref[rows];
  for (int q = tid; q < total_missing; q += kPlanThreads) {
    int lo = 0, hi = rows - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_mpref[mid] <= q) lo = mid; else hi = mid - 1;
    }
    const int row = lo;
    int wl = 0, wh = W - 1;
    while (wl < wh) {
      const int mid = (wl + wh + 1) >> 1;
      if (s_wpref[mid] <= q) wl = mid; else wh = mid - 1;
    }
    const int page = wl * 32 + select_bit(a.st.bitmap[wl], q - s_wpref[wl]);
    const int j = q - s_mpref[row];
    a.pending[row * pstride + 1 + j] = page;
    const int pos = s_kvpref[row] + s_owned[row] + j;
    if (pos < a.kv_capacity) a.kv_indices[pos] = page;
  }
  __syncthreads();
  for (int q = tid; q < total_missing; q += kPlanThreads) {
    int lo = 0, hi = rows - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_mpref[mid] <= q) lo = mid; else hi = mid - 1;
    }
    const int page = a.pending[lo * pstride + 1 + (q - s_mpref[lo])];
    atomicAnd(&a.st.bitmap[page >> 5], ~(1u << (page & 31)));
  }
  __threadfence_block();
  __syncthreads();

  // owned pages, padding pages, per-token slots: one warp per row
  const int warp = tid >> 5, lane = tid & 31;
  for (int row = warp; row < rows; row += kPlanThreads / 32) {
    const int kvp = s_kvpref[row];
    const int s = s_slot[row];
    if (s_real[row]) {
      const int32_t* tab = a.st.table + static_cast<int64_t>(s) * a.max_pages;
      const int own = s_owned[row];
      for (int j = lane; j < own; j += 32)
        if (kvp + j < a.kv_capacity) a.kv_indices[kvp + j] = tab[j];
      const int L = s_len[row];
      const int tp = s_tpref[row];
      const int ps = a.st.pos_start[s];
      for (int i = lane; a.positions != nullptr && i < s_adv[row]; i += 32) {
        const int abs = L + i;
        const int pi = abs / P;
        const int page = pi < own ? tab[pi] : a.pending[row * pstride + 1 + (pi - own)];
        if (tp + i < a.token_capacity) {
          a.write_pages[tp + i] = page;
          a.write_offsets[tp + i] = abs % P;
          a.positions[tp + i] = ps + i;
        }
      }
    } else if (lane == 0) {
      int sp = -1;
      if (row < a.scratch_count) sp = a.scratch[row]; else report(a.status, NQT_DEV_CAPACITY);
      if (kvp < a.kv_capacity) a.kv_indices[kvp] = sp < 0 ? 0 : sp;
      if (!a.prefill && a.positions != nullptr) {
        const int tp = s_tpref[row];
        if (tp < a.token_capacity) {
          a.write_pages[tp] = sp < 0 ? 0 : sp;
          a.write_offsets[tp] = 0;
          a.positions[tp] = 0;
        }
      }
    }
  }
  // spare token slots on the scratch pages
  const int real_tokens = s_real_tokens;
  for (int t = s_tpref[rows] + tid; a.positions != nullptr && t < a.token_capacity; t += kPlanThreads) {
    const int slot_i = t - real_tokens;
    const int sp_idx = slot_i / P;
    int sp = 0;
    if (sp_idx < a.scratch_count && slot_i >= 0) sp = a.scratch[sp_idx]; else report(a.status, NQT_DEV_CAPACITY);
    a.write_pages[t] = sp;
    a.write_offsets[t] = slot_i >= 0 ? slot_i % P : 0;
    a.positions[t] = 0;
  }
}

__global__ void planner_init_kernel(StateView st, int total_pages, int slots, int scratch_count) {
  const int W = (total_pages + 31) / 32;
  for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < W; w += gridDim.x * blockDim.x) {
    uint32_t m = 0;
    for (int b = 0; b < 32; ++b) {
      const int page = w * 32 + b;
      if (page >= scratch_count && page < total_pages) m |= 1u << b;
    }
    st.bitmap[w] = m;
  }
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < slots; s += gridDim.x * blockDim.x) {
    st.seq_len[s] = 0;
    st.pos_start[s] = 0;
    st.n_pages[s] = 0;
  }
}

__global__ void plan_commit_kernel(StateView st, int total_pages, int slots, int max_pages, const int32_t* row_slot,
                                   const int32_t* row_adv, const int32_t* row_publish, int rows,
                                   int32_t* pending, int32_t* status) {
  const int pstride = max_pages + 1;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const int s = row_slot[r];
    const int missing = pending[r * pstride];
    if (s < 0 || missing < 0) continue;  // padding row or a row the plan did not reserve
    if (s >= slots) {
      report(status, NQT_DEV_BAD_SLOT);
      continue;
    }
    pending[r * pstride] = -1;  // consumed: a second commit of the same plan is a no-op
    if (row_publish[r] != 0) {
      const int owned = st.n_pages[s];
      if (owned + missing > max_pages) {
        report(status, NQT_DEV_TABLE_FULL);
        continue;
      }
      for (int j = 0; j < missing; ++j) st.table[static_cast<int64_t>(s) * max_pages + owned + j] = pending[r * pstride + 1 + j];
      st.n_pages[s] = owned + missing;
      st.seq_len[s] += row_adv[r];
      st.pos_start[s] += row_adv[r];
    } else {
      for (int j = 0; j < missing; ++j) {
        const int page = pending[r * pstride + 1 + j];
        if (page >= 0 && page < total_pages) atomicOr(&st.bitmap[page >> 5], 1u << (page & 31));
      }
    }
  }
}

__global__ void plan_release_kernel(StateView st, int total_pages, int slots, int max_pages, const int32_t* list,
                                    int count, int32_t* status) {
  // one block per listed slot
  const int i = blockIdx.x;
  if (i >= count) return;
  const int s = list[i];
  if (s < 0 || s >= slots) {
    if (threadIdx.x == 0) report(status, NQT_DEV_BAD_SLOT);
    return;
  }
  const int n = st.n_pages[s];
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const int page = st.table[static_cast<int64_t>(s) * max_pages + j];
    if (page >= 0 && page < total_pages) atomicOr(&st.bitmap[page >> 5], 1u << (page & 31));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    st.n_pages[s] = 0;
    st.seq_len[s] = 0;
    st.pos_start[s] = 0;
  }
}

__global__ void plan_import_kernel(StateView st, int total_pages, int max_pages, int slot, const int32_t* pages,
                                   int n, int seq_len, int pos_start, int32_t* status) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
    const int page = pages[j];
    if (page < 0 || page >= total_pages) {
      report(status, NQT_DEV_BAD_PAGE);
      continue;
    }
    st.table[static_cast<int64_t>(slot) * max_pages + j] = page;
    atomicAnd(&st.bitmap[page >> 5], ~(1u << (page & 31)));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    st.n_pages[slot] = n;
    st.seq_len[slot] = seq_len;
    st.pos_start[slot] = pos_start;
  }
}

}  // namespace
}  // namespace nqt

using namespace nqt;

extern "C" size_t nqt_planner_state_bytes(int total_pages, int slots, int max_pages_per_slot) {
  if (total_pages < 1 || slots < 1 || max_pages_per_slot < 1) return 0;
  return state_bytes(total_pages, slots, max_pages_per_slot);
}

extern "C" int nqt_planner_init(void* state, int total_pages, int slots, int max_pages_per_slot, int scratch_count,
                                void* stream) {
  if (!state || total_pages < 1 || slots < 1 || max_pages_per_slot < 1) return NQT_ERR_ARG;
  if (scratch_count < 0 || scratch_count > total_pages) return NQT_ERR_ARG;
  const StateView v = state_view(state, total_pages, slots, max_pages_per_slot);
  const int W = (total_pages + 31) / 32;
  const int work = W > slots ? W : slots;
  planner_init_kernel<<<(work + 255) / 256, 256, 0, as_stream(stream)>>>(v, total_pages, slots, scratch_count);
  return check_launch("planner_init");
}

extern "C" int nqt_plan_step(void* state, int total_pages, int slots, int max_pages_per_slot, int page_size,
                             const int32_t* row_slot, const int32_t* row_advance, int capture_rows,
                             int token_capacity, const int32_t* scratch_pages, int scratch_count, int prefill,
                             int32_t* qo_indptr, int32_t* kv_indptr, int32_t* kv_indices, int kv_indices_capacity,
                             int32_t* last_page_len, int64_t* position_ids, int64_t* write_pages,
                             int64_t* write_offsets, int32_t* pending, void* decode_workspace,
                             size_t decode_workspace_bytes, int num_qo_heads, int head_dim, int32_t* status,
                             void* stream) {
  if (!state || !row_slot || !row_advance || !scratch_pages || !kv_indptr || !kv_indices || !last_page_len ||
      !pending)
    return NQT_ERR_ARG;
  // allocation-only step: no per-token metadata at all
  const bool tokens_out = position_ids != nullptr;
  if (tokens_out != (write_pages != nullptr) || tokens_out != (write_offsets != nullptr)) return NQT_ERR_ARG;
  if (!tokens_out) token_capacity = 0;
  if (prefill && tokens_out && !qo_indptr) return NQT_ERR_ARG;

  if (capture_rows < 1 || capture_rows > kMaxRows || (tokens_out && token_capacity < 1) || page_size < 1)
    return NQT_ERR_ARG;
  if (total_pages < 1 || slots < 1 || max_pages_per_slot < 1 || scratch_count < 0) return NQT_ERR_ARG;
  const int W = (total_pages + 31) / 32;
  if (W > kMaxWordsSmem) return NQT_ERR_UNSUPPORTED;
  PlanArgs a;
  a.st = state_view(state, total_pages, slots, max_pages_per_slot);
  a.total_pages = total_pages;
  a.slots = slots;
  a.max_pages = max_pages_per_slot;
  a.page_size = page_size;
  a.row_slot = row_slot;
  a.row_adv = row_advance;
  a.rows = capture_rows;
  a.token_capacity = token_capacity;
  a.scratch = scratch_pages;
  a.scratch_count = scratch_count;
  a.prefill = prefill;
  a.qo_indptr = prefill ? qo_indptr : nullptr;  // may be NULL for an allocation-only step
  a.kv_indptr = kv_indptr;
  a.kv_indices = kv_indices;
  a.kv_capacity = kv_indices_capacity;
  a.last_len = last_page_len;
  a.positions = position_ids;
  a.write_pages = write_pages;
  a.write_offsets = write_offsets;
  a.pending = pending;
  a.status = status;
  const size_t smem = 4 * static_cast<size_t>(W + 1);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(plan_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * (kMaxWordsSmem + 1));
    configured = true;
  }
  cudaStream_t s = as_stream(stream);
  plan_step_kernel<<<1, kPlanThreads, smem, s>>>(a);
  int rc = check_launch("plan_step");
  if (rc != NQT_OK || decode_workspace == nullptr) return rc;
  return nqt_decode_plan(kv_indptr, last_page_len, capture_rows, capture_rows, page_size, num_qo_heads, head_dim,
                         decode_workspace, decode_workspace_bytes, stream);
}

extern "C" int nqt_plan_commit(void* state, int total_pages, int slots, int max_pages_per_slot,
                               const int32_t* row_slot, const int32_t* row_advance, const int32_t* row_publish,
                               int capture_rows, int32_t* pending, int32_t* status, void* stream) {
  if (!state || !row_slot || !row_advance || !row_publish || !pending || capture_rows < 1) return NQT_ERR_ARG;
  const StateView v = state_view(state, total_pages, slots, max_pages_per_slot);
  plan_commit_kernel<<<(capture_rows + 127) / 128, 128, 0, as_stream(stream)>>>(
      v, total_pages, slots, max_pages_per_slot, row_slot, row_advance, row_publish, capture_rows, pending, status);
  return check_launch("plan_commit");
}

extern "C" int nqt_plan_release(void* state, int total_pages, int slots, int max_pages_per_slot,
                                const int32_t* slot_list, int count, int32_t* status, void* stream) {
  if (!state || !slot_list || count < 0) return NQT_ERR_ARG;
  if (count == 0) return NQT_OK;
  const StateView v = state_view(state, total_pages, slots, max_pages_per_slot);
  plan_release_kernel<<<count, 256, 0, as_stream(stream)>>>(v, total_pages, slots, max_pages_per_slot, slot_list,
                                                            count, status);
  return check_launch("plan_release");
}

extern "C" int nqt_plan_import(void* state, int total_pages, int slots, int max_pages_per_slot, int slot,
                               const int32_t* pages, int n_pages, int seq_len, int pos_start, int32_t* status,
                               void* stream) {
  if (!state || (n_pages > 0 && !pages) || slot < 0 || slot >= slots) return NQT_ERR_ARG;
  if (n_pages < 0 || n_pages > max_pages_per_slot || seq_len < 0) return NQT_ERR_ARG;
  const StateView v = state_view(state, total_pages, slots, max_pages_per_slot);
  plan_import_kernel<<<1, 256, 0, as_stream(stream)>>>(v, total_pages, max_pages_per_slot, slot, pages, n_pages,
                                                       seq_len, pos_start, status);
  return check_launch("plan_import");
}
