// GPU SparseAttnSharedkvMetadata scheduler (sm_100a), bit-identical to the
// reference port sparse_attn_sharedkv_tilelang/metadata.py.
//
// One CTA of 1024 threads:
//   phase 1 (all threads): per-batch split info (metadata.py:671-683) and
//     per-row costs (metadata.py:428-667) summed into per-batch cost / block
//     counts and the batch's last-block cost (metadata.py:685-714). Rows are
//     cut into 32-row items spread over the warps.
//   phase 2 (warp 0): the greedy core assignment (metadata.py:872-923) with
//     AssignByBatch (718-745) and AssignByRow (747-764). The row walk is done
//     32 rows at a time: each lane evaluates one row, a warp scan gives the
//     running core cost, and a ballot finds the first row that breaks the
//     tolerance test -- the same decision sequence as the sequential loop.
//     Rows past a batch's end are evaluated with the same formulas, which is
//     how the reference behaves when the row cursor overruns the batch.
//   phase 3: pack faMetadata / fdMetadata (metadata.py:974-1009).
#include "sas_common.cuh"

namespace {

using i128 = __int128;
constexpr int kThreads = 1024;
constexpr int64_t kInt64Max = 0x7fffffffffffffffLL;
constexpr int64_t kRowScanCap = 1LL << 24;

struct MetaArgs {
  const int32_t* cu_q;
  const int32_t* cu_kv;
  const int32_t* sq;
  const int32_t* skv;
  int n_cu_q, n_cu_kv, n_sq, n_skv;
  int64_t batch, max_q, max_kv, nq, nkv, cmp_topk, cmp_ratio, mask_mode, win_left;
  int layout_q, layout_kv, has_cmp, aic;
  // derived (metadata.py:359-389)
  int64_t pre_token, next_token, group, m_base, s2_base;
  int is_s1g, is_cfa, is_scfa, att_mode;
};

struct BatchInfo {
  i128 pre_lu, next_lu;
  int64_t s1, s2, s1g_base, s1g_tail;
  int64_t cost, block, lbc;
  long long last_row;  // last row index with a non-zero block count (-1 = none)
  int64_t r0_cost, r0_block, r0_lbc, r0_s2start;
};

struct RowInfo {
  int64_t cost, block, lbc, s2_start;
};

__device__ int64_t s1_size(const MetaArgs& A, int64_t b) {
  if (A.n_sq > 0) return A.sq[b];
  if (A.layout_q == SAS_LAYOUT_TND && A.n_cu_q > 0) return (int64_t)A.cu_q[b + 1] - A.cu_q[b];
  return A.max_q;
}
__device__ int64_t s2_size(const MetaArgs& A, int64_t b) {
  if (A.n_skv > 0) return A.skv[b];
  if (A.layout_kv == SAS_LAYOUT_TND && A.n_cu_kv > 0) return (int64_t)A.cu_kv[b + 1] - A.cu_kv[b];
  return A.max_kv;
}

__device__ __forceinline__ int64_t calc_cost(int64_t m, int64_t s2) {
  return 6 * ((m + 15) >> 4) + 10 * ((s2 + 63) >> 6);
}

// _calc_s1g_cache (metadata.py:634-667) reduced to the fields the assignment reads.
__device__ RowInfo row_info(const MetaArgs& A, const BatchInfo& bi, int64_t idx) {
  RowInfo r{0, 0, 0, 0};
  if (bi.s1g_base == 0) return r;  // early return path: everything zero
  // _calc_s2_token_range (479-501)
  i128 first, last;
  if (bi.s1 == 0 || bi.s2 == 0) {
    first = 0;
    last = 0;
  } else if (!A.att_mode) {
    first = 0;
    last = bi.s2 - 1;
  } else {
    int64_t g_first = idx * A.m_base;
    int64_t lim = bi.s1 * A.group;
    int64_t g_last = (g_first + A.m_base < lim ? g_first + A.m_base : lim) - 1;
    int64_t f, l;
    if (A.is_s1g) {
      f = sas::floordiv64(g_first, A.group);
      l = sas::floordiv64(g_last, A.group);
    } else if (sas::floordiv64(g_first, bi.s1) == sas::floordiv64(g_last, bi.s1)) {
      f = g_first - sas::floordiv64(g_first, bi.s1) * bi.s1;
      l = g_last - sas::floordiv64(g_last, bi.s1) * bi.s1;
    } else {
      f = 0;
      l = bi.s1;
    }
    first = (i128)f - bi.pre_lu;
    last = (i128)l + bi.next_lu;
  }
  // _calc_block_range_and_tail_size (512-547)
  int64_t of = 0, ol = 0, win_end = 0, win_tail = 0;
  if (!(first >= bi.s2 || last < 0 || last < first)) {
    of = (int64_t)(first < 0 ? (i128)0 : (first > bi.s2 - 1 ? (i128)(bi.s2 - 1) : first));
    ol = (int64_t)(last < 0 ? (i128)0 : (last > bi.s2 - 1 ? (i128)(bi.s2 - 1) : last));
    win_end = sas::floordiv64(ol - of, A.s2_base) + 1;
    int64_t t = ol - of + 1;
    win_tail = t - sas::floordiv64(t, A.s2_base) * A.s2_base;
  }
  int64_t cmp_start = win_end;
  int64_t last_tok = (A.has_cmp && A.cmp_ratio > 0) ? sas::floordiv64(ol + 1, A.cmp_ratio) : 0;
  int64_t act = 0;
  if (A.is_cfa) act = last_tok;
  else if (A.is_scfa) act = last_tok < A.cmp_topk ? last_tok : A.cmp_topk;
  int64_t cmp_end = act == 0 ? cmp_start : cmp_start + sas::floordiv64(act - 1, A.s2_base) + 1;
  int64_t cmp_tail = act - sas::floordiv64(act, A.s2_base) * A.s2_base;
  // cost table (440-477) and win / cmp caches (549-621)
  int64_t s1t = bi.s1g_tail;
  bool tail_row = (idx == bi.s1g_base - 1) && s1t != 0;
  int64_t nn = calc_cost(A.m_base, A.s2_base);
  int64_t tn = s1t == 0 ? 0 : calc_cost(s1t, A.s2_base);
  int64_t w_nt = win_tail == 0 ? 0 : calc_cost(A.m_base, win_tail);
  int64_t w_tt = (s1t == 0 || win_tail == 0) ? 0 : calc_cost(s1t, win_tail);
  int64_t c_nt = cmp_tail == 0 ? 0 : calc_cost(A.m_base, cmp_tail);
  int64_t c_tt = (s1t == 0 || cmp_tail == 0) ? 0 : calc_cost(s1t, cmp_tail);
  int64_t win_block = 0, win_cost = 0, win_lbc = 0;
  if (0 < win_end) {
    win_block = win_end;
    int64_t t = win_tail != 0 ? 1 : 0, n = win_block - t;
    if (tail_row) {
      win_cost = tn * n + w_tt * t;
      win_lbc = t > 0 ? w_tt : tn;
    } else {
      win_cost = nn * n + w_nt * t;
      win_lbc = t > 0 ? w_nt : nn;
    }
  }
  int64_t cmp_block = 0, cmp_cost = 0, cmp_lbc = 0;
  if (cmp_start < cmp_end) {
    // the cmp entries of the cost table are only (re)computed when has_cmp
    cmp_block = cmp_end - cmp_start;
    int64_t t = cmp_tail != 0 ? 1 : 0, n = cmp_block - t;
    if (tail_row) {
      cmp_cost = tn * n + c_tt * t;
      cmp_lbc = t > 0 ? c_tt : tn;
    } else {
      cmp_cost = nn * n + c_nt * t;
      cmp_lbc = t > 0 ? c_nt : nn;
    }
  }
  // _gather_win_and_cmp (623-632)
  r.s2_start = win_block > 0 ? 0 : cmp_start;
  r.lbc = cmp_block > 0 ? cmp_lbc : win_lbc;
  r.block = win_block + cmp_block;
  r.cost = win_cost + cmp_cost;
  return r;
}

__device__ void batch_info_init(const MetaArgs& A, int64_t b, BatchInfo& bi) {
  bi.s1 = s1_size(A, b);
  bi.s2 = s2_size(A, b);
  bi.pre_lu = (A.mask_mode == 4) ? (i128)bi.s1 - bi.s2 + A.pre_token : (i128)A.pre_token;
  if (A.mask_mode == 0 || A.mask_mode == 1 || A.mask_mode == 2) bi.next_lu = A.next_token;
  else if (A.mask_mode == 3) bi.next_lu = (i128)bi.s2 - bi.s1;
  else if (A.mask_mode == 4) bi.next_lu = (i128)bi.s2 - bi.s1 + A.next_token;
  else bi.next_lu = A.next_token;
  int64_t rows = bi.s1 * A.group;
  bi.s1g_base = sas::floordiv64(rows + A.m_base - 1, A.m_base);
  bi.s1g_tail = rows - sas::floordiv64(rows, A.m_base) * A.m_base;
  bi.cost = bi.block = bi.lbc = 0;
  bi.last_row = -1;
}

__device__ __forceinline__ int64_t warp_incl_scan(int64_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int64_t u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  return v;
}
__device__ __forceinline__ int64_t warp_sum(int64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(kThreads, 1)
    sas_metadata_kernel(MetaArgs A, BatchInfo* __restrict__ binfo, long long* __restrict__ item_prefix,
                        int64_t* __restrict__ core_out, int32_t* __restrict__ meta_out, int32_t* status) {
  __shared__ long long s_max_cost;
  __shared__ int s_all_zero;
  __shared__ int64_t s_used;
  __shared__ long long s_total_items;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t B = A.batch;
  if (tid == 0) {
    s_max_cost = 0;
    s_all_zero = 1;
    s_used = 1;
  }
  __syncthreads();
  // ---- phase 1a: split info per batch (metadata.py:671-683)
  for (int64_t b = tid; b < B; b += kThreads) {
    BatchInfo bi;
    batch_info_init(A, b, bi);
    int64_t s2b = sas::floordiv64(bi.s2 + A.s2_base - 1, A.s2_base);
    if (bi.s1g_base != 0 && s2b != 0) s_all_zero = 0;
    binfo[b] = bi;
  }
  __syncthreads();
  if (s_all_zero) {
    // metadata.py:959-964
    if (tid == 0) {
      core_out[0] = B * A.nkv;
      core_out[1] = 0;
      core_out[2] = 0;
      s_used = 1;
    }
  } else {
    // ---- phase 1b: per-batch costs over 32-row items (metadata.py:685-714)
    // item counts per batch, exclusive prefix (single-warp scan over batches)
    if (warp == 0) {
      long long carry = 0;
      for (int64_t b0 = 0; b0 < B; b0 += 32) {
        int64_t b = b0 + lane;
        long long n = 0;
        if (b < B) {
          const BatchInfo& bi = binfo[b];
          if (bi.s1 != 0 && bi.s2 != 0) n = (bi.s1g_base + 31) >> 5;
        }
        long long inc = warp_incl_scan(n, lane);
        if (b < B) item_prefix[b] = carry + inc - n;
        carry += __shfl_sync(0xffffffffu, inc, 31);
      }
      if (lane == 0) {
        item_prefix[B] = carry;
        s_total_items = carry;
      }
    }
    __syncthreads();
    const long long n_items = s_total_items;
    for (long long it = warp; it < n_items; it += kThreads / 32) {
      // batch of this item: last b with item_prefix[b] <= it
      int64_t lo = 0, hi = B - 1;
      while (lo < hi) {
        int64_t mid = (lo + hi + 1) >> 1;
        if (item_prefix[mid] <= it) lo = mid; else hi = mid - 1;
      }
      const int64_t b = lo;
      const BatchInfo bi = binfo[b];
      int64_t row = (it - item_prefix[b]) * 32 + lane;
      RowInfo r{0, 0, 0, 0};
      if (row < bi.s1g_base) r = row_info(A, bi, row);
      int64_t cs = warp_sum(r.cost), bs = warp_sum(r.block);
      long long mx = r.cost;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        long long u = __shfl_xor_sync(0xffffffffu, mx, o);
        mx = u > mx ? u : mx;
      }
      long long lr = (row < bi.s1g_base && r.block > 0) ? row : -1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        long long u = __shfl_xor_sync(0xffffffffu, lr, o);
        lr = u > lr ? u : lr;
      }
      if (lane == 0) {
        atomicAdd(reinterpret_cast<unsigned long long*>(&binfo[b].cost), (unsigned long long)cs);
        atomicAdd(reinterpret_cast<unsigned long long*>(&binfo[b].block), (unsigned long long)bs);
        atomicMax(&s_max_cost, mx);
        if (lr >= 0) atomicMax(&binfo[b].last_row, lr);
      }
    }
    __syncthreads();
    for (int64_t b = tid; b < B; b += kThreads) {
      BatchInfo bi = binfo[b];
      if (bi.last_row >= 0) bi.lbc = row_info(A, bi, bi.last_row).lbc;
      RowInfo r0 = row_info(A, bi, 0);
      bi.r0_cost = r0.cost;
      bi.r0_block = r0.block;
      bi.r0_lbc = r0.lbc;
      bi.r0_s2start = r0.s2_start;
      binfo[b] = bi;
    }
    __syncthreads();
    // ---- phase 2: greedy assignment (metadata.py:898-923), warp 0
    if (warp == 0 && A.aic > 0) {
      int64_t total = 0;
      for (int64_t b = lane; b < B; b += 32) total += binfo[b].cost * A.nkv;
      total = warp_sum(total);
      const int64_t max_s1g_cost = s_max_cost;
      int64_t cur_b = 0, cur_bn2 = 0, cur_s1g = 0, cur_s2 = 0, cur_core = 0;
      int64_t unassigned = total;
      int64_t bn2_cost = binfo[0].cost, bn2_block = binfo[0].block;
      RowInfo sc{binfo[0].r0_cost, binfo[0].r0_block, binfo[0].r0_lbc, binfo[0].r0_s2start};
      cur_s2 = sc.s2_start;
      bool finished = false, overrun = false;
      const int64_t nbn2 = B * A.nkv;
      for (int64_t i = 0; i < A.aic; ++i) {
        if (finished || unassigned <= 0) break;
        cur_core = i;
        int64_t den = A.aic - cur_core;
        if (den < 1) den = 1;
        int64_t avg = sas::floordiv64(unassigned, den);
        const int64_t limit = avg > max_s1g_cost ? avg : max_s1g_cost;
        int64_t core_cost = 0;
        // AssignByBatch (718-745): sequential over batches (uniform in the warp)
        while (bn2_cost == 0 || limit + (binfo[cur_b].lbc >> 1) >= core_cost + bn2_cost) {
          core_cost += bn2_cost;
          cur_bn2 += 1;
          if (cur_bn2 == nbn2) {
            cur_s1g = 0;
            cur_s2 = 0;
            finished = true;
            break;
          }
          int64_t nb = sas::floordiv64(cur_bn2, A.nkv);
          if (nb != cur_b) cur_b = nb;
          const BatchInfo& bi = binfo[cur_b];
          bn2_cost = bi.cost;
          bn2_block = bi.block;
          cur_s1g = 0;
          sc = RowInfo{bi.r0_cost, bi.r0_block, bi.r0_lbc, bi.r0_s2start};
          cur_s2 = sc.s2_start;
        }
        if (!finished) {
          // AssignByRow (747-764)
          const BatchInfo bi = binfo[cur_b];
          if (limit + (sc.lbc >> 1) >= core_cost + sc.cost) {
            // take the current row, then walk the following non-empty rows
            core_cost += sc.cost;
            bn2_cost = bn2_cost - sc.cost < 0 ? 0 : bn2_cost - sc.cost;
            bn2_block = bn2_block - sc.block < 0 ? 0 : bn2_block - sc.block;
            int64_t base = cur_s1g + 1;
            int64_t scanned = 0;
            while (true) {
              RowInfo r = row_info(A, bi, base + lane);
              const bool considered = r.block != 0;
              const int64_t c = considered ? r.cost : 0;
              const int64_t incl = warp_incl_scan(c, lane);
              const int64_t excl = incl - c;
              const bool ok = limit + (r.lbc >> 1) >= core_cost + excl + r.cost;
              const unsigned fail = __ballot_sync(0xffffffffu, considered && !ok);
              if (fail) {
                const int f = __ffs(fail) - 1;
                const int64_t took = __shfl_sync(0xffffffffu, excl, f);
                const int64_t blk_before = warp_incl_scan(considered && lane < f ? r.block : 0, lane);
                const int64_t took_blk = __shfl_sync(0xffffffffu, blk_before, 31);
                core_cost += took;
                bn2_cost = bn2_cost - took < 0 ? 0 : bn2_cost - took;
                bn2_block = bn2_block - took_blk < 0 ? 0 : bn2_block - took_blk;
                cur_s1g = base + f;
                sc.cost = __shfl_sync(0xffffffffu, r.cost, f);
                sc.block = __shfl_sync(0xffffffffu, r.block, f);
                sc.lbc = __shfl_sync(0xffffffffu, r.lbc, f);
                sc.s2_start = __shfl_sync(0xffffffffu, r.s2_start, f);
                cur_s2 = sc.s2_start;
                break;
              }
              const int64_t all = __shfl_sync(0xffffffffu, incl, 31);
              const int64_t all_blk = warp_sum(considered ? r.block : 0);
              core_cost += all;
              bn2_cost = bn2_cost - all < 0 ? 0 : bn2_cost - all;
              bn2_block = bn2_block - all_blk < 0 ? 0 : bn2_block - all_blk;
              base += 32;
              scanned += 32;
              if (scanned > kRowScanCap) {
                overrun = true;
                break;
              }
            }
            if (overrun) break;
          }
        }
        if (lane == 0) {
          core_out[3 * i + 0] = cur_bn2;
          core_out[3 * i + 1] = cur_s1g;
          core_out[3 * i + 2] = cur_s2;
        }
        unassigned -= core_cost;
      }
      if (overrun && lane == 0 && status) atomicCAS(status, 0, SAS_ERR_SCHED_OVERRUN);
      if (lane == 0) s_used = cur_core + 1 < 1 ? 1 : cur_core + 1;
      (void)bn2_block;
    }
  }
  __syncthreads();
  // ---- phase 3: pack (metadata.py:974-1009)
  const int64_t used = s_used;
  for (int i = tid; i < SAS_META_SIZE; i += kThreads) meta_out[i] = 0;
  __syncthreads();
  if (tid < SAS_AIC_CORE_NUM) {
    const int i = tid;
    int32_t* row = meta_out + i * 8;
    if (!(i >= used || i >= A.aic)) {
      row[0] = 1;
      row[1] = (int32_t)(i == 0 ? 0 : core_out[3 * (i - 1) + 0]);
      row[2] = (int32_t)(i == 0 ? 0 : core_out[3 * (i - 1) + 1]);
      row[3] = (int32_t)(i == 0 ? 0 : core_out[3 * (i - 1) + 2]);
      row[4] = (int32_t)core_out[3 * i + 0];
      row[5] = (int32_t)core_out[3 * i + 1];
      row[6] = (int32_t)core_out[3 * i + 2];
    }
  }
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace

extern "C" size_t sas_metadata_workspace_bytes(int32_t batch_size, int32_t aic_core_num) {
  size_t b = batch_size > 0 ? (size_t)batch_size : 1;
  size_t c = aic_core_num > 0 ? (size_t)aic_core_num : 1;
  return align_up(sizeof(BatchInfo) * b, 256) + align_up(sizeof(long long) * (b + 1), 256) +
         align_up(sizeof(int64_t) * 3 * c, 256);
}

extern "C" int sas_metadata(const int32_t* cu_seqlens_q, int32_t n_cu_seqlens_q, const int32_t* cu_seqlens_ori_kv,
                            int32_t n_cu_seqlens_ori_kv, const int32_t* seqused_q, int32_t n_seqused_q,
                            const int32_t* seqused_kv, int32_t n_seqused_kv, int32_t batch_size,
                            int32_t max_seqlen_q, int32_t max_seqlen_kv, int32_t num_heads_q,
                            int32_t num_heads_kv, int32_t head_dim, int32_t cmp_topk, int32_t cmp_ratio,
                            int32_t ori_mask_mode, int32_t ori_win_left, int32_t layout_q, int32_t layout_kv,
                            int32_t has_cmp_kv, int32_t aic_core_num, int32_t* metadata_out, int32_t* status,
                            void* workspace, size_t workspace_bytes, void* stream) {
  (void)head_dim;
  if (!metadata_out) return SAS_ERR_INVALID_ARG;
  if (!sas::select_device_of(metadata_out)) return SAS_ERR_INVALID_ARG;
  MetaArgs A{};
  A.cu_q = n_cu_seqlens_q > 0 ? cu_seqlens_q : nullptr;
  A.cu_kv = n_cu_seqlens_ori_kv > 0 ? cu_seqlens_ori_kv : nullptr;
  A.sq = n_seqused_q > 0 ? seqused_q : nullptr;
  A.skv = n_seqused_kv > 0 ? seqused_kv : nullptr;
  A.n_cu_q = A.cu_q ? n_cu_seqlens_q : 0;
  A.n_cu_kv = A.cu_kv ? n_cu_seqlens_ori_kv : 0;
  A.n_sq = A.sq ? n_seqused_q : 0;
  A.n_skv = A.skv ? n_seqused_kv : 0;
  A.layout_q = layout_q;
  A.layout_kv = layout_kv;
  // batch size resolution (metadata.py:345-350)
  int64_t B = batch_size;
  if (A.n_sq > 0) B = A.n_sq;
  else if (layout_q == SAS_LAYOUT_TND && A.n_cu_q > 0) B = A.n_cu_q - 1;
  if (B < 0) return SAS_ERR_INVALID_ARG;
  // every per-batch read must stay inside the arrays the caller passed
  if (A.n_sq == 0 && layout_q == SAS_LAYOUT_TND && A.n_cu_q > 0 && A.n_cu_q < B + 1) return SAS_ERR_INVALID_ARG;
  if (A.n_skv > 0 && A.n_skv < B) return SAS_ERR_INVALID_ARG;
  if (A.n_skv == 0 && layout_kv == SAS_LAYOUT_TND && A.n_cu_kv > 0 && A.n_cu_kv < B + 1) return SAS_ERR_INVALID_ARG;
  if (num_heads_kv <= 0 || num_heads_q / num_heads_kv <= 0 || aic_core_num < 0) return SAS_ERR_INVALID_ARG;
  if (has_cmp_kv && cmp_ratio == 0) return SAS_ERR_INVALID_ARG;
  A.batch = B;
  A.max_q = max_seqlen_q;
  A.max_kv = max_seqlen_kv;
  A.nq = num_heads_q;
  A.nkv = num_heads_kv;
  A.cmp_topk = cmp_topk;
  A.cmp_ratio = cmp_ratio;
  A.mask_mode = ori_mask_mode;
  A.win_left = ori_win_left;
  A.has_cmp = has_cmp_kv != 0;
  A.aic = aic_core_num;
  // _params_init (metadata.py:359-389)
  if (ori_mask_mode == 0) {
    A.pre_token = kInt64Max;
    A.next_token = kInt64Max;
    A.att_mode = 0;
  } else if (ori_mask_mode == 3) {
    A.pre_token = kInt64Max;
    A.next_token = 0;
    A.att_mode = 1;
  } else {
    A.pre_token = ori_win_left > -1 ? ori_win_left : kInt64Max;
    A.next_token = 0;
    A.att_mode = 1;
  }
  A.is_s1g = (layout_q == SAS_LAYOUT_BSND || layout_q == SAS_LAYOUT_TND || layout_q == SAS_LAYOUT_BSH);
  A.group = num_heads_q / num_heads_kv;
  A.is_cfa = A.is_scfa = 0;
  if (A.has_cmp) {
    if (cmp_topk > 0) A.is_scfa = 1;
    else A.is_cfa = 1;
  }
  A.m_base = A.group;
  A.s2_base = 512;
  const size_t need = sas_metadata_workspace_bytes((int32_t)(B > 0 ? B : 1), aic_core_num);
  if (!workspace || workspace_bytes < need) return SAS_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  const size_t b1 = (size_t)(B > 0 ? B : 1);
  BatchInfo* binfo = reinterpret_cast<BatchInfo*>(ws);
  long long* item_prefix = reinterpret_cast<long long*>(ws + align_up(sizeof(BatchInfo) * b1, 256));
  int64_t* core_out = reinterpret_cast<int64_t*>(ws + align_up(sizeof(BatchInfo) * b1, 256) +
                                                 align_up(sizeof(long long) * (b1 + 1), 256));
  sas_metadata_kernel<<<1, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(A, binfo, item_prefix, core_out,
                                                                             metadata_out, status);
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}
