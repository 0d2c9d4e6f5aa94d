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
#include <mutex>

#include "sas_common.cuh"

namespace {

using i128 = __int128;
constexpr int kThreads = 512;
constexpr int kSmemCap = 200 * 1024;  // dynamic shared memory of the scheduler CTA
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
  int64_t scan_cap;  // rows the greedy walk may scan past a core's start before it reports an overrun
  int fast;  // row_info_fast applies (band mask, finite window, S1G layout)
  int smem;  // dynamic shared memory of this launch, bytes
};

struct BatchInfo {
  i128 pre_lu, next_lu;
  int64_t s1, s2, s1g_base, s1g_tail;
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

// Division-free form of row_info for the configuration the attention API
// uses: band mask with a finite left window (mode 4, win_left >= 0), an S1G
// query layout (BSND / TND / BSH), and every length below 2^30. There
// m_base == group, so row idx covers exactly query token idx (clamped to the
// last token when the cursor runs past the batch), and the s2 range is
// [idx + s2 - s1 - win_left, min(idx, s1-1) + s2 - s1].
__device__ __forceinline__ bool row_fast_ok(const MetaArgs& A, const BatchInfo& bi, int64_t idx) {
  return A.fast && bi.s1 < (1 << 30) && bi.s2 < (1 << 30) && idx < (1LL << 30);
}

__device__ RowInfo row_info_fast(const MetaArgs& A, const BatchInfo& bi, int64_t idx) {
  RowInfo r{0, 0, 0, 0};
  if (bi.s1g_base == 0) return r;
  const int64_t s1 = bi.s1, s2 = bi.s2;
  int64_t first, last;
  if (s2 == 0) {
    first = 0;
    last = 0;
  } else {
    const int64_t s1_last = idx < s1 ? idx : s1 - 1;
    first = idx - (s1 - s2 + A.win_left);
    last = s1_last + (s2 - s1);
  }
  int64_t ol = 0, win_end = 0, win_tail = 0;
  if (!(first >= s2 || last < 0 || last < first)) {
    const int64_t of = first < 0 ? 0 : (first > s2 - 1 ? s2 - 1 : first);
    ol = last > s2 - 1 ? s2 - 1 : last;
    win_end = ((ol - of) >> 9) + 1;
    win_tail = (ol - of + 1) & 511;
  }
  const int64_t cmp_start = win_end;
  int64_t act = 0;
  if (A.has_cmp && A.cmp_ratio > 0) {
    const int64_t last_tok = (int64_t)((uint32_t)(ol + 1) / (uint32_t)A.cmp_ratio);
    if (A.is_cfa) act = last_tok;
    else if (A.is_scfa) act = last_tok < A.cmp_topk ? last_tok : A.cmp_topk;
  }
  const int64_t cmp_end = act == 0 ? cmp_start : cmp_start + ((act - 1) >> 9) + 1;
  const int64_t cmp_tail = act & 511;
  // s1g tail is zero (m_base == group), so only the "normal" rows of the
  // cost table (metadata.py:449-477) are used
  const int64_t nn = calc_cost(A.m_base, 512);
  int64_t win_block = 0, win_cost = 0, win_lbc = 0;
  if (win_end > 0) {
    win_block = win_end;
    const int64_t t = win_tail != 0 ? 1 : 0;
    const int64_t w_nt = t ? calc_cost(A.m_base, win_tail) : 0;
    win_cost = nn * (win_block - t) + w_nt * t;
    win_lbc = t ? w_nt : nn;
  }
  int64_t cmp_block = 0, cmp_cost = 0, cmp_lbc = 0;
  if (cmp_start < cmp_end) {
    cmp_block = cmp_end - cmp_start;
    const int64_t t = cmp_tail != 0 ? 1 : 0;
    const int64_t c_nt = t ? calc_cost(A.m_base, cmp_tail) : 0;
    cmp_cost = nn * (cmp_block - t) + c_nt * t;
    cmp_lbc = t ? c_nt : nn;
  }
  r.s2_start = win_block > 0 ? 0 : cmp_start;
  r.lbc = cmp_block > 0 ? cmp_lbc : win_lbc;
  r.block = win_block + cmp_block;
  r.cost = win_cost + cmp_cost;
  return r;
}

// _calc_s1g_cache (metadata.py:634-667) reduced to the fields the assignment reads.
__device__ __noinline__ RowInfo row_info_general(const MetaArgs& A, const BatchInfo& bi, int64_t idx) {
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

__device__ __forceinline__ RowInfo row_info(const MetaArgs& A, const BatchInfo& bi, int64_t idx) {
  return row_fast_ok(A, bi, idx) ? row_info_fast(A, bi, idx) : row_info_general(A, bi, idx);
}

__device__ __forceinline__ BatchInfo make_bi(const MetaArgs& A, int64_t s1, int64_t s2) {
  BatchInfo bi;
  bi.s1 = s1;
  bi.s2 = s2;
  bi.pre_lu = (A.mask_mode == 4) ? (i128)s1 - s2 + A.pre_token : (i128)A.pre_token;
  if (A.mask_mode == 0 || A.mask_mode == 1 || A.mask_mode == 2) bi.next_lu = A.next_token;
  else if (A.mask_mode == 3) bi.next_lu = (i128)s2 - s1;
  else if (A.mask_mode == 4) bi.next_lu = (i128)s2 - s1 + A.next_token;
  else bi.next_lu = A.next_token;
  // m_base == group (metadata.py:388), so every s1g row is one query token
  bi.s1g_base = s1 > 0 ? s1 : 0;
  bi.s1g_tail = 0;
  return bi;
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

// Per-batch state, structure of arrays. It lives in shared memory when the
// batch fits (kSmemBatches), else in the caller's workspace; same code.
constexpr int kSmemBatches = 2048;
constexpr int64_t kSmallRows = 8;  // batches with at most this many rows are costed by one thread
constexpr int kNumArrays = 9;  // s1, s2, cost, lbc, last_row, r0 cost, r0 lbc, r0 block, item prefix (+1)
struct Arrays {
  long long *s1, *s2, *cost, *lbc, *last_row, *r0c, *r0l, *r0b, *item;
  __device__ void bind(long long* base, int64_t B) {
    s1 = base;
    s2 = s1 + B;
    cost = s2 + B;
    lbc = cost + B;
    last_row = lbc + B;
    r0c = last_row + B;
    r0l = r0c + B;
    r0b = r0l + B;
    item = r0b + B;  // B + 1 entries
  }
};

// Smallest j in [lo, hi) with val(j) > x, for val non-decreasing on [lo, hi);
// hi when there is none. One warp, 32 probes per round.
template <typename I, typename F>
__device__ __forceinline__ I warp_first_gt(const F& val, I lo, I hi, I x, int lane) {
  while (hi > lo) {
    const I step = (hi - lo + 31) / 32;
    const I pk = lo + (I)(lane + 1) * step - 1;
    const bool gt = pk >= hi || val(pk) > x;
    const unsigned bal = __ballot_sync(0xffffffffu, gt);
    if (bal == 0) return hi;
    const int k0 = __ffs(bal) - 1;
    const I p0 = lo + (I)(k0 + 1) * step - 1;
    lo = lo + (I)k0 * step;
    hi = p0 < hi ? p0 : hi;
  }
  return lo;
}

// Inclusive prefix sums of in[0, n) into out (a different array), by the
// whole block: each thread sums a contiguous run, the runs are scanned
// through shared memory, then each thread writes its run.
template <typename F>
__device__ void block_inclusive_prefix(const F& in, long long* out, int64_t n, long long* s_warp) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kWarps = kThreads / 32;
  const int64_t per = (n + kThreads - 1) / kThreads;
  const int64_t b0 = (int64_t)tid * per, b1 = b0 + per < n ? b0 + per : n;
  long long local = 0;
  for (int64_t b = b0; b < b1; ++b) local += in(b);
  long long incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    long long w = lane < kWarps ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long u = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += u;
    }
    if (lane < kWarps) s_warp[lane] = w;
  }
  __syncthreads();
  long long run = (warp ? s_warp[warp - 1] : 0) + incl - local;
  for (int64_t b = b0; b < b1; ++b) {
    run += in(b);
    out[b] = run;
  }
  __syncthreads();
}

template <typename I>
struct RowT {
  I cost, block, lbc, s2_start;
};
template <typename I>
__device__ __forceinline__ I warp_scan_t(I v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const I u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  return v;
}

// The greedy core assignment (metadata.py:872-923) run by one warp. I is
// int when every cost sum is known to fit in 31 bits (checked by the caller),
// which halves the shuffle chain of the serial walk; else long long.
template <typename I>
__device__ void assign_cores(const MetaArgs& A, const Arrays& V, int64_t B, int64_t total, long long max_cost,
                             int lane, int64_t* core_out, bool& overrun, int64_t& used, const int2* rc,
                             const long long* pitem, const long long* pcost) {
      const I max_s1g_cost = (I)max_cost;
  I cur_b = 0, cur_bn2 = 0, cur_s1g = 0, cur_s2 = 0, cur_core = 0;
  I unassigned = (I)total;
  I bn2_cost = (I)V.cost[0];
  RowT<I> sc{(I)V.r0c[0], (I)V.r0b[0], (I)V.r0l[0], 0};
  cur_s2 = sc.s2_start;
  bool finished = false;
  const I nbn2 = (I)(B * A.nkv);
  for (int i = 0; i < A.aic; ++i) {
    if (finished || unassigned <= 0) break;
    cur_core = i;
    I den = (I)A.aic - cur_core;
    if (den < 1) den = 1;
    const I avg = unassigned / den;  // both positive here
    const I limit = avg > max_s1g_cost ? avg : max_s1g_cost;
    I core_cost = 0;
    // AssignByBatch (718-745): the current bn2 is tested with its remaining
    // cost, every following bn2 with its batch's full cost. With P the
    // inclusive prefix of bn2 costs, bn2 j >= base stops the walk when
    // c_j != 0 and P(j) - lbc_j/2 > thr := limit - core_cost + P(base-1).
    // Since lbc_j <= c_j, every non-empty j after the first j with
    // P(j) > thr stops it too, so the stop is that j or the next non-empty
    // one: two prefix searches instead of a walk.
    if (bn2_cost == 0 || limit + ((I)V.lbc[cur_b] >> 1) >= core_cost + bn2_cost) {
      core_cost += bn2_cost;
      const I nkv = (I)A.nkv;
      auto pbn = [&](I j) -> I {  // inclusive prefix of bn2 costs
        if (nkv == 1) return (I)pcost[j];
        const I b = j / nkv;
        return nkv * (b > 0 ? (I)pcost[b - 1] : (I)0) + (j - b * nkv + 1) * (I)V.cost[b];
      };
      const I base = cur_bn2 + 1;
      const I pb0 = pbn(base - 1);
      const I thr = limit - core_cost + pb0;
      // the first 32 bn2s directly (the usual case), the rest by search
      I jf;
      {
        const I j = base + lane;
        bool stop = j >= nbn2;
        if (!stop) {
          const I bj = nkv == 1 ? j : j / nkv;
          stop = (I)V.cost[bj] != 0 && pbn(j) - ((I)V.lbc[bj] >> 1) > thr;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, stop);
        if (bal) {
          jf = base + (I)(__ffs(bal) - 1);
          if (jf > nbn2) jf = nbn2;
        } else {
          jf = warp_first_gt<I>(pbn, base + 32, nbn2, thr, lane);
          if (jf < nbn2) {
            const I bj = nkv == 1 ? jf : jf / nkv;
            if (!((I)V.cost[bj] != 0 && pbn(jf) - ((I)V.lbc[bj] >> 1) > thr))
              jf = warp_first_gt<I>(pbn, jf + 1, nbn2, pbn(jf), lane);
          }
        }
      }
      core_cost += (jf > base ? pbn(jf - 1) : pb0) - pb0;  // the bn2s in [base, jf)
      if (jf >= nbn2) {
        cur_bn2 = nbn2;
        cur_s1g = 0;
        cur_s2 = 0;
        finished = true;
      } else {
        cur_bn2 = jf;
        cur_b = nkv == 1 ? jf : jf / nkv;
        bn2_cost = (I)V.cost[cur_b];
        cur_s1g = 0;
        sc = RowT<I>{(I)V.r0c[cur_b], (I)V.r0b[cur_b], (I)V.r0l[cur_b], 0};
        cur_s2 = 0;
      }
    }
    if (!finished) {
      // AssignByRow (747-764)
      if (limit + (sc.lbc >> 1) >= core_cost + sc.cost) {
        const BatchInfo bi = make_bi(A, V.s1[cur_b], V.s2[cur_b]);
        // take the current row, then walk the following non-empty rows
        core_cost += sc.cost;
        bn2_cost = bn2_cost - sc.cost < 0 ? 0 : bn2_cost - sc.cost;
        I base = cur_s1g + 1;
        int64_t scanned = 0;
        bool done = false;
        if (rc != nullptr && bi.s1g_base > kSmallRows && (int64_t)base < bi.s1g_base) {
          // cached rows [base, s1g_base): prefix search as in AssignByBatch
          // (a row has blocks exactly when its cost is non-zero, and its lbc
          // never exceeds its cost)
          const long long it0 = V.item[cur_b];
          auto pex = [&](long long it) -> long long { return pitem[it] - rc[it * 32 + 31].x; };
          const long long b0x = pex(it0);
          auto prow = [&](I row) -> I {  // inclusive prefix of the batch's row costs
            const long long it = it0 + (row >> 5);
            return (I)(pex(it) - b0x + rc[it * 32 + (row & 31)].x);
          };
          auto crow = [&](I row) -> I { return row > 0 ? prow(row) - prow(row - 1) : prow(row); };
          const I end = (I)bi.s1g_base;
          const I pr0 = prow(base - 1);
          const I thr = limit - core_cost + pr0;
          auto rfail = [&](I row) -> bool {
            const I lbc = (I)rc[(it0 + (row >> 5)) * 32 + (row & 31)].y;
            return crow(row) != 0 && prow(row) - (lbc >> 1) > thr;
          };
          I rf;
          {
            const I row = base + lane;
            const unsigned bal = __ballot_sync(0xffffffffu, row < end && rfail(row));
            if (bal) {
              rf = base + (I)(__ffs(bal) - 1);
            } else {
              rf = warp_first_gt<I>(prow, base + 32 < end ? base + 32 : end, end, thr, lane);
              if (rf < end && !rfail(rf)) rf = warp_first_gt<I>(prow, rf + 1, end, prow(rf), lane);
            }
          }
          const I took = (rf > base ? prow(rf - 1) : pr0) - pr0;
          core_cost += took;
          bn2_cost = bn2_cost - took < 0 ? 0 : bn2_cost - took;
          if (rf < end) {
            cur_s1g = rf;
            const I c = crow(rf);
            sc = RowT<I>{c, (I)(c != 0), (I)rc[(it0 + (rf >> 5)) * 32 + (rf & 31)].y, 0};
            cur_s2 = 0;
            done = true;
          } else {
            scanned = (int64_t)(end - base);
            base = end;  // continue past the batch's rows (metadata.py walks on)
          }
        }
        while (!done) {
          const int64_t row = (int64_t)base + lane;
          const RowInfo r64 = row_info(A, bi, row);
          RowT<I> r{(I)r64.cost, (I)r64.block, (I)r64.lbc, (I)r64.s2_start};
          const bool considered = r.block != 0;
          const I c = considered ? r.cost : 0;
          const I incl = warp_scan_t<I>(c, lane);
          const I excl = incl - c;
          const bool ok = limit + (r.lbc >> 1) >= core_cost + excl + r.cost;
          const unsigned fail = __ballot_sync(0xffffffffu, considered && !ok);
          if (fail) {
            const int f = __ffs(fail) - 1;
            const I took = __shfl_sync(0xffffffffu, excl, f);
            core_cost += took;
            bn2_cost = bn2_cost - took < 0 ? 0 : bn2_cost - took;
            cur_s1g = base + f;
            sc.cost = __shfl_sync(0xffffffffu, r.cost, f);
            sc.block = __shfl_sync(0xffffffffu, r.block, f);
            sc.lbc = __shfl_sync(0xffffffffu, r.lbc, f);
            sc.s2_start = __shfl_sync(0xffffffffu, r.s2_start, f);
            cur_s2 = sc.s2_start;
            break;
          }
          const I all = __shfl_sync(0xffffffffu, incl, 31);
          core_cost += all;
          bn2_cost = bn2_cost - all < 0 ? 0 : bn2_cost - all;
          base += 32;
          scanned += 32;
          if (scanned > A.scan_cap) {
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
  used = cur_core + 1 < 1 ? 1 : cur_core + 1;
}

__global__ void __launch_bounds__(kThreads, 1)
    sas_metadata_kernel(MetaArgs A, long long* __restrict__ ws_arrays, int64_t* __restrict__ core_out,
                        int32_t* __restrict__ meta_out, int32_t* status) {
  extern __shared__ long long sh_arrays[];
  sas::pdl_launch_dependents();  // the plan kernel that follows may start launching

  __shared__ long long s_max_cost;
  __shared__ int s_all_zero;
  __shared__ int64_t s_used;
  __shared__ long long s_total_items;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t B = A.batch;
  Arrays V;
  V.bind(B <= kSmemBatches ? sh_arrays : ws_arrays, B > 0 ? B : 1);
  if (tid == 0) {
    s_max_cost = 0;
    s_all_zero = 1;
    s_used = 1;
  }
  __syncthreads();
  // ---- phase 1a: split info per batch (metadata.py:671-683)
  for (int64_t b = tid; b < B; b += kThreads) {
    const int64_t s1 = s1_size(A, b), s2 = s2_size(A, b);
    V.s1[b] = s1;
    V.s2[b] = s2;
    const BatchInfo bi = make_bi(A, s1, s2);
    const int64_t s2b = sas::floordiv64(s2 + A.s2_base - 1, A.s2_base);
    if (bi.s1g_base != 0 && s2b != 0) s_all_zero = 0;
    V.cost[b] = 0;
    V.last_row[b] = -1;
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
    if (warp == 0) {
      long long carry = 0;
      for (int64_t b0 = 0; b0 < B; b0 += 32) {
        const int64_t b = b0 + lane;
        long long n = 0;
        if (b < B) {
          const long long s1 = V.s1[b], s2 = V.s2[b];
          if (s1 != 0 && s2 != 0) {
            const int64_t rows = make_bi(A, s1, s2).s1g_base;
            n = rows <= kSmallRows ? 0 : (rows + 31) >> 5;  // small batches: one thread each
          }
        }
        const long long inc = warp_incl_scan(n, lane);
        if (b < B) V.item[b] = carry + inc - n;
        carry += __shfl_sync(0xffffffffu, inc, 31);
      }
      if (lane == 0) {
        V.item[B] = carry;
        s_total_items = carry;
      }
    }
    __syncthreads();
    const long long n_items = s_total_items;
    // per-row cost cache for the serial walk, in shared memory after the batch arrays
    const size_t arr_bytes = B <= kSmemBatches ? sizeof(long long) * (kNumArrays * (size_t)(B > 0 ? B : 1) + 1) : 0;
    // per row (prefix of the row costs within its 32-row item, lbc), then one
    // inclusive prefix of item totals per item
    int2* rc = nullptr;
    long long* pitem = nullptr;
    if (A.fast && arr_bytes + 16 + (size_t)n_items * (32 * sizeof(int2) + sizeof(long long)) <= (size_t)A.smem) {
      rc = reinterpret_cast<int2*>(reinterpret_cast<char*>(sh_arrays) + ((arr_bytes + 15) & ~(size_t)15));
      pitem = reinterpret_cast<long long*>(rc + n_items * 32);
    }
    for (long long it = warp; it < n_items; it += kThreads / 32) {
      int64_t lo = 0, hi = B - 1;  // batch of this item: last b with item[b] <= it
      while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (V.item[mid] <= it) lo = mid; else hi = mid - 1;
      }
      const int64_t b = lo;
      const BatchInfo bi = make_bi(A, V.s1[b], V.s2[b]);
      const int64_t row = (it - V.item[b]) * 32 + lane;
      RowInfo r{0, 0, 0, 0};
      if (row < bi.s1g_base) r = row_info(A, bi, row);
      const int64_t incl = warp_incl_scan(r.cost, lane);
      if (rc) rc[it * 32 + lane] = make_int2((int)incl, (int)r.lbc);
      const int64_t cs = __shfl_sync(0xffffffffu, incl, 31);
      long long mx = r.cost;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const long long u = __shfl_xor_sync(0xffffffffu, mx, o);
        mx = u > mx ? u : mx;
      }
      long long lr = (row < bi.s1g_base && r.block > 0) ? row : -1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const long long u = __shfl_xor_sync(0xffffffffu, lr, o);
        lr = u > lr ? u : lr;
      }
      if (lane == 0) {
        atomicAdd(reinterpret_cast<unsigned long long*>(&V.cost[b]), (unsigned long long)cs);
        atomicMax(&s_max_cost, mx);
        if (lr >= 0) atomicMax(&V.last_row[b], lr);
      }
    }
    __syncthreads();
    for (int64_t b = tid; b < B; b += kThreads) {
      const BatchInfo bi = make_bi(A, V.s1[b], V.s2[b]);
      if (bi.s1 != 0 && bi.s2 != 0 && bi.s1g_base <= kSmallRows) {
        // small batch (decode): all its rows here, in row order
        long long cost = 0, mx = 0, lr = -1;
        for (int64_t row = 0; row < bi.s1g_base; ++row) {
          const RowInfo r = row_info(A, bi, row);
          cost += r.cost;
          mx = r.cost > mx ? r.cost : mx;
          if (r.block > 0) lr = row;
        }
        V.cost[b] = cost;
        V.last_row[b] = lr;
        atomicMax(&s_max_cost, mx);
      }
      V.lbc[b] = V.last_row[b] >= 0 ? row_info(A, bi, V.last_row[b]).lbc : 0;
      const RowInfo r0 = row_info(A, bi, 0);  // its s2 start is always block 0
      V.r0c[b] = r0.cost;
      V.r0l[b] = r0.lbc;
      V.r0b[b] = r0.block;
    }
    __syncthreads();
    // inclusive prefix of the batch costs, into last_row's storage (dead now)
    __shared__ long long s_scan[kThreads / 32];
    block_inclusive_prefix([&](int64_t b) { return V.cost[b]; }, V.last_row, B, s_scan);
    // row cache: inclusive prefix of the item totals (rc.x is the prefix within an item)
    if (rc) block_inclusive_prefix([&](int64_t it) { return (long long)rc[it * 32 + 31].x; }, pitem, n_items, s_scan);
    // ---- phase 2: greedy assignment (metadata.py:898-923), warp 0
    if (warp == 0 && A.aic > 0) {
      int64_t total = 0;
      for (int64_t b = lane; b < B; b += 32) total += V.cost[b] * A.nkv;
      total = warp_sum(total);
      bool overrun = false;
      int64_t used = 1;
      if (A.fast && total < (1LL << 30) && s_max_cost < (1LL << 30) && B * A.nkv < (1LL << 30))
        assign_cores<int>(A, V, B, total, s_max_cost, lane, core_out, overrun, used, rc, pitem, V.last_row);
      else
        assign_cores<long long>(A, V, B, total, s_max_cost, lane, core_out, overrun, used, rc, pitem, V.last_row);
      if (overrun && lane == 0 && status) atomicCAS(status, 0, SAS_ERR_SCHED_OVERRUN);
      if (lane == 0) s_used = used;
    }
  }
  __syncthreads();
  // ---- phase 3: pack (metadata.py:974-1009)
  const int64_t used = s_used;
  for (int i = tid; i < SAS_META_SIZE; i += kThreads) {
    int32_t v = 0;
    if (i < SAS_AIC_CORE_NUM * 8) {
      const int core = i >> 3, f = i & 7;
      if (core < used && core < A.aic) {
        if (f == 0) v = 1;
        else if (f <= 3) v = core == 0 ? 0 : (int32_t)core_out[3 * (core - 1) + (f - 1)];
        else if (f <= 6) v = (int32_t)core_out[3 * core + (f - 4)];
      }
    }
    meta_out[i] = v;
  }
}


// ---------------------------------------------------------------------------
// Flash-decode (supportFd) variant of the scheduler: metadata.py with the
// scheduler's supportFd flag set, which the reference declares and never
// turns on (metadata.py:323-325). It differs from the default schedule in
// four places: a core's cost limit is the plain average (not raised to the
// largest row, 884-887), a core may end inside a row after the row walk
// (AssignByBlock, 777-794; a core that took nothing is given one block,
// 859-870, with the cursor rules of 829-857), a row cut between cores is
// recorded as a flash-decode head (796-827), and the heads are spread over
// the vector cores (925-954) into fdMetadata[72][8] (995-1009).
// Phase 1 (per-batch costs) runs on the whole block, one thread per row;
// the greedy walk is sequential by nature and runs on one thread.

// Every field of _calc_s1g_cache (metadata.py:634-667) that the flash-decode
// walk reads. With m_base == group the s1g tail is always zero, so only the
// "normal" rows of the cost table apply.
struct RowD {
  int64_t cost, block, lbc, s2_start, s2_end, cmp_s2_start, win_nbc, win_lbc, cmp_nbc, cmp_lbc;
};

__device__ RowD row_detail(const MetaArgs& A, const BatchInfo& bi, int64_t idx) {
  RowD r{};
  if (bi.s1g_base == 0) return r;  // metadata.py:641-652: every field read here is zero
  i128 first, last;
  if (bi.s1 == 0 || bi.s2 == 0) {
    first = 0;
    last = 0;
  } else if (!A.att_mode) {
    first = 0;
    last = bi.s2 - 1;
  } else {
    const int64_t g_first = idx * A.m_base;
    const int64_t lim = bi.s1 * A.group;
    const int64_t g_last = (g_first + A.m_base < lim ? g_first + A.m_base : lim) - 1;
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
  int64_t ol = 0, win_end = 0, win_tail = 0;
  if (!(first >= bi.s2 || last < 0 || last < first)) {
    const int64_t of = (int64_t)(first < 0 ? (i128)0 : (first > bi.s2 - 1 ? (i128)(bi.s2 - 1) : first));
    ol = (int64_t)(last < 0 ? (i128)0 : (last > bi.s2 - 1 ? (i128)(bi.s2 - 1) : last));
    win_end = sas::floordiv64(ol - of, A.s2_base) + 1;
    const int64_t t = ol - of + 1;
    win_tail = t - sas::floordiv64(t, A.s2_base) * A.s2_base;
  }
  const int64_t cmp_start = win_end;
  const int64_t last_tok = (A.has_cmp && A.cmp_ratio > 0) ? sas::floordiv64(ol + 1, A.cmp_ratio) : 0;
  int64_t act = 0;
  if (A.is_cfa) act = last_tok;
  else if (A.is_scfa) act = last_tok < A.cmp_topk ? last_tok : A.cmp_topk;
  const int64_t cmp_end = act == 0 ? cmp_start : cmp_start + sas::floordiv64(act - 1, A.s2_base) + 1;
  const int64_t cmp_tail = act - sas::floordiv64(act, A.s2_base) * A.s2_base;
  const int64_t nn = calc_cost(A.m_base, A.s2_base);
  int64_t win_block = 0, win_cost = 0;
  if (0 < win_end) {
    win_block = win_end;
    const int64_t t = win_tail != 0 ? 1 : 0;
    const int64_t w_nt = t ? calc_cost(A.m_base, win_tail) : 0;
    win_cost = nn * (win_block - t) + w_nt * t;
    r.win_lbc = t ? w_nt : nn;
    r.win_nbc = nn;
  }
  int64_t cmp_block = 0, cmp_cost = 0;
  if (cmp_start < cmp_end) {
    cmp_block = cmp_end - cmp_start;
    const int64_t t = cmp_tail != 0 ? 1 : 0;
    const int64_t c_nt = t ? calc_cost(A.m_base, cmp_tail) : 0;
    cmp_cost = nn * (cmp_block - t) + c_nt * t;
    r.cmp_lbc = t ? c_nt : nn;
    r.cmp_nbc = nn;
  }
  r.cmp_s2_start = cmp_start;
  r.s2_start = win_block > 0 ? 0 : cmp_start;
  if (cmp_block > 0) {
    r.lbc = r.cmp_lbc;
    r.s2_end = cmp_end;
  } else {
    r.lbc = r.win_lbc;
    r.s2_end = win_end;
  }
  r.block = win_block + cmp_block;
  r.cost = win_cost + cmp_cost;
  return r;
}

constexpr int kFdHeads = SAS_AIC_CORE_NUM + 64;  // flash-decode heads (at most one per core boundary)
constexpr int kFdVec = 72 + 64;                   // vector cores

__global__ void __launch_bounds__(kThreads, 1)
    sas_metadata_fd_kernel(MetaArgs A, int64_t aiv, long long* __restrict__ ws, int64_t* __restrict__ core_out,
                           int32_t* __restrict__ meta_out, int32_t* status) {
  sas::pdl_launch_dependents();
  __shared__ int s_all_zero;
  __shared__ long long s_max_cost, s_total;
  __shared__ int64_t s_used, s_nvec;
  __shared__ int64_t f_bn2[kFdHeads], f_m[kFdHeads], f_ws[kFdHeads], f_split[kFdHeads], f_msz[kFdHeads];
  __shared__ int64_t v_idx[kFdVec], v_mstart[kFdVec], v_mnum[kFdVec];
  const int tid = threadIdx.x;
  const int64_t B = A.batch;
  const int64_t B1 = B > 0 ? B : 1;
  long long* cost = ws;           // per batch: cost, blocks, last row with blocks, row prefix
  long long* blocks = cost + B1;
  long long* last_row = blocks + B1;
  long long* rows = last_row + B1;  // B + 1: rows before batch b
  if (tid == 0) {
    s_all_zero = 1;
    s_max_cost = 0;
    s_total = 0;
    s_used = 1;
    s_nvec = 0;
  }
  __syncthreads();
  // split info (metadata.py:671-683); a batch's rows are costed only when
  // both of its lengths are non-zero (metadata.py:687-689)
  for (int64_t b = tid; b < B; b += kThreads) {
    const int64_t s1 = s1_size(A, b), s2 = s2_size(A, b);
    const BatchInfo bi = make_bi(A, s1, s2);
    const int64_t s2b = sas::floordiv64(s2 + A.s2_base - 1, A.s2_base);
    if (bi.s1g_base != 0 && s2b != 0) s_all_zero = 0;
    cost[b] = 0;
    blocks[b] = 0;
    last_row[b] = -1;
    rows[b] = (s1 == 0 || s2 == 0) ? 0 : bi.s1g_base;
  }
  __syncthreads();
  if (tid == 0) {  // exclusive prefix of the costed rows (small batches: one pass)
    long long run = 0;
    for (int64_t b = 0; b < B; ++b) {
      const long long n = rows[b];
      rows[b] = run;
      run += n;
    }
    rows[B] = run;
  }
  __syncthreads();
  if (!s_all_zero) {
    // per-row costs (metadata.py:685-714), one thread per row
    const long long nrows = rows[B];
    for (long long r = tid; r < nrows; r += kThreads) {
      int64_t lo = 0, hi = B - 1;  // last batch with rows[b] <= r
      while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (rows[mid] <= r) lo = mid;
        else hi = mid - 1;
      }
      const int64_t b = lo, row = r - rows[b];
      const BatchInfo bi = make_bi(A, s1_size(A, b), s2_size(A, b));
      const RowD d = row_detail(A, bi, row);
      atomicAdd(reinterpret_cast<unsigned long long*>(&cost[b]), (unsigned long long)d.cost);
      atomicAdd(reinterpret_cast<unsigned long long*>(&blocks[b]), (unsigned long long)d.block);
      atomicMax(&s_max_cost, (long long)d.cost);
      if (d.block > 0) atomicMax(&last_row[b], (long long)row);
    }
    __syncthreads();
    if (tid == 0) {
      // the greedy walk (metadata.py:872-923) with the flash-decode steps
      for (int64_t b = 0; b < B; ++b) s_total += cost[b] * A.nkv;
      auto lbc_of = [&](int64_t b) -> int64_t {  // bn2_last_block_cost_of_each_batch
        if (last_row[b] < 0) return 0;
        return row_detail(A, make_bi(A, s1_size(A, b), s2_size(A, b)), last_row[b]).lbc;
      };
      int64_t cur_b = 0, cur_bn2 = 0, cur_s1g = 0, cur_s2 = 0, cur_core = 0;
      int64_t unassigned = s_total, bn2_cost = cost[0], bn2_block = blocks[0];
      int64_t split_part = 1;
      const int64_t fd_data_num = 1;  // never advanced in metadata.py
      int64_t n_head = 0;
      bool finished = false, overrun = false;
      BatchInfo bi = make_bi(A, s1_size(A, 0), s2_size(A, 0));
      RowD sc = row_detail(A, bi, 0);
      cur_s2 = sc.s2_start;
      auto new_row = [&](int64_t idx) {
        cur_s1g = idx;
        sc = row_detail(A, bi, idx);
      };
      auto block_cost = [&]() -> int64_t {  // metadata.py:766-775
        if (cur_s2 < sc.cmp_s2_start) return cur_s2 == sc.cmp_s2_start - 1 ? sc.win_lbc : sc.win_nbc;
        return cur_s2 == sc.s2_end - 1 ? sc.cmp_lbc : sc.cmp_nbc;
      };
      for (int64_t i = 0; i < A.aic; ++i) {
        if (finished || unassigned <= 0) break;
        cur_core = i;
        const int64_t den = A.aic - cur_core > 1 ? A.aic - cur_core : 1;
        const int64_t limit = sas::floordiv64(unassigned, den);
        int64_t ccost = 0, cblock = 0;
        // AssignByBatch (718-745)
        while (!finished && (bn2_cost == 0 || limit + sas::floordiv64(lbc_of(cur_b), 2) >= ccost + bn2_cost)) {
          ccost += bn2_cost;
          cblock += bn2_block;
          cur_bn2 += 1;
          if (cur_bn2 == B * A.nkv) {
            cur_s1g = 0;
            cur_s2 = 0;
            finished = true;
            break;
          }
          if (sas::floordiv64(cur_bn2, A.nkv) != cur_b) {
            cur_b = sas::floordiv64(cur_bn2, A.nkv);
            bi = make_bi(A, s1_size(A, cur_b), s2_size(A, cur_b));
          }
          bn2_cost = cost[cur_b];
          bn2_block = blocks[cur_b];
          new_row(0);
          cur_s2 = sc.s2_start;
        }
        // AssignByRow (747-764)
        if (!finished) {
          int64_t scanned = 0;
          while (limit + sas::floordiv64(sc.lbc, 2) >= ccost + sc.cost) {
            ccost += sc.cost;
            cblock += sc.block;
            bn2_cost = bn2_cost - sc.cost < 0 ? 0 : bn2_cost - sc.cost;
            bn2_block = bn2_block - sc.block < 0 ? 0 : bn2_block - sc.block;
            do {
              new_row(cur_s1g + 1);
              if (++scanned > A.scan_cap) overrun = true;
            } while (sc.block == 0 && !overrun);
            cur_s2 = sc.s2_start;
            if (overrun) break;
          }
        }
        if (overrun) break;
        // AssignByBlock (777-794)
        if (!finished) {
          int64_t c = block_cost();
          int64_t scanned = 0;
          while (limit + sas::floordiv64(c, 2) >= ccost + c) {
            ccost += c;
            cblock += 1;
            cur_s2 += 1;
            bn2_cost -= c;
            sc.cost -= c;
            bn2_block -= 1;
            sc.block -= 1;
            c = block_cost();
            if (++scanned > A.scan_cap) {
              overrun = true;
              break;
            }
          }
        }
        if (overrun) break;
        // ForceAssign (859-870) with UpdateCursor (829-857)
        if (cblock == 0 && !finished) {
          const int64_t c = block_cost();
          ccost += c;
          cblock += 1;
          cur_s2 += 1;
          bn2_cost -= c;
          bn2_block -= 1;
          sc.cost -= c;
          sc.block -= 1;
          bool upd_row = false, upd_b = false;
          if (cur_s2 >= sc.s2_end) {
            cur_s2 = 0;
            cur_s1g += 1;
            upd_row = true;
          }
          if (cur_s1g >= bi.s1g_base) {
            cur_s1g = 0;
            cur_bn2 += 1;
          }
          if (cur_bn2 == B * A.nkv) {
            cur_s1g = 0;
            cur_s2 = 0;
            finished = true;
          } else {
            if (sas::floordiv64(cur_bn2, A.nkv) != cur_b) {
              cur_b = sas::floordiv64(cur_bn2, A.nkv);
              cur_s1g = 0;
              upd_b = true;
              upd_row = true;
            }
            if (upd_b) {
              bi = make_bi(A, s1_size(A, cur_b), s2_size(A, cur_b));
              bn2_cost = cost[cur_b];
              bn2_block = blocks[cur_b];
            }
            if (upd_row) {
              new_row(cur_s1g);
              cur_s2 = 0;  // win_s2_start, always 0
            }
          }
        }
        core_out[3 * i + 0] = cur_bn2;
        core_out[3 * i + 1] = cur_s1g;
        core_out[3 * i + 2] = cur_s2;
        unassigned -= ccost;
        // a row cut between this core and the one before (796-827)
        if (cur_core != 0 && split_part > 1 &&
            !(cur_bn2 == core_out[3 * (i - 1)] && cur_s1g == core_out[3 * (i - 1) + 1])) {
          if (n_head >= A.aic || n_head >= kFdHeads) {
            overrun = true;
            break;
          }
          const int64_t sb = sas::floordiv64(core_out[3 * (i - 1)], A.nkv);
          const int64_t srow = core_out[3 * (i - 1) + 1];
          const BatchInfo sbi = make_bi(A, s1_size(A, sb), s2_size(A, sb));
          f_bn2[n_head] = core_out[3 * (i - 1)];
          f_m[n_head] = srow;
          f_ws[n_head] = fd_data_num - split_part;
          f_split[n_head] = split_part;
          f_msz[n_head] = srow == sbi.s1g_base - 1 ? sbi.s1 * A.group - srow * A.m_base : A.m_base;
          n_head += 1;
          split_part = 1;
        }
        if (sc.s2_start < cur_s2 && cur_s2 <= sc.s2_end) split_part += 1;
      }
      if (overrun && status) atomicCAS(status, 0, SAS_ERR_SCHED_OVERRUN);
      s_used = cur_core + 1;
      // the heads over the vector cores (925-954)
      long long total_fd = 0;
      for (int64_t h = 0; h < n_head; ++h) total_fd += f_split[h] * f_msz[h];
      const int64_t avg = aiv > 0 ? sas::floordiv64(total_fd, aiv) : 0;
      int64_t cur = 0;
      if (n_head > 0 && avg > 0) {
        for (int64_t h = 0; h < n_head; ++h) {
          const int64_t nv = sas::floordiv64(f_split[h] * f_msz[h], avg);
          if (nv == 0) continue;
          const int64_t ave = sas::floordiv64(f_msz[h], nv);
          for (int64_t v = 0; v < nv; ++v) {
            if (cur >= aiv || cur >= kFdVec) break;
            v_idx[cur] = h;
            v_mstart[cur] = v * ave;
            v_mnum[cur] = v < nv - 1 ? ave : f_msz[h] - v * ave;
            ++cur;
          }
        }
      }
      s_nvec = cur;
    }
  } else if (tid == 0) {  // metadata.py:959-964
    core_out[0] = B * A.nkv;
    core_out[1] = 0;
    core_out[2] = 0;
  }
  __syncthreads();
  // pack (metadata.py:974-1009)
  const int64_t used = s_used, nvec = s_nvec;
  for (int i = tid; i < SAS_META_SIZE; i += kThreads) {
    int32_t v = 0;
    if (i < SAS_AIC_CORE_NUM * 8) {
      const int core = i >> 3, f = i & 7;
      if (core < used && core < A.aic) {
        if (f == 0) v = 1;
        else if (f <= 3) v = core == 0 ? 0 : (int32_t)core_out[3 * (core - 1) + (f - 1)];
        else if (f <= 6) v = (int32_t)core_out[3 * core + (f - 4)];
      }
    } else {
      const int j = i - SAS_AIC_CORE_NUM * 8, vc = j >> 3, f = j & 7;
      if (vc < nvec && vc < aiv) {
        const int64_t h = v_idx[vc];
        switch (f) {
          case 0: v = 1; break;
          case 1: v = (int32_t)f_bn2[h]; break;
          case 2: v = (int32_t)f_m[h]; break;
          case 3: v = (int32_t)f_ws[h]; break;
          case 4: v = (int32_t)f_split[h]; break;
          case 5: v = (int32_t)v_mstart[vc]; break;
          case 6: v = (int32_t)v_mnum[vc]; break;
          default: v = 0;
        }
      }
    }
    meta_out[i] = v;
  }
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

long long g_scan_cap = kRowScanCap;  // SAS_OPT_SCHED_SCAN_CAP

}  // namespace

namespace sas {
void set_sched_scan_cap(long long cap) { g_scan_cap = cap > 0 ? cap : kRowScanCap; }
}  // namespace sas

extern "C" size_t sas_metadata_workspace_bytes(int32_t batch_size, int32_t aic_core_num) {
  const size_t b = batch_size > 0 ? (size_t)batch_size : 1;
  const size_t c = aic_core_num > 0 ? (size_t)aic_core_num : 1;
  return align_up(sizeof(long long) * (kNumArrays * b + 1), 256) + align_up(sizeof(int64_t) * 3 * c, 256);
}

namespace {
int metadata_launch(const int32_t* cu_seqlens_q, int32_t n_cu_seqlens_q, const int32_t* cu_seqlens_ori_kv,
                            int32_t n_cu_seqlens_ori_kv, const int32_t* seqused_q, int32_t n_seqused_q,
                            const int32_t* seqused_kv, int32_t n_seqused_kv, int32_t batch_size,
                            int32_t max_seqlen_q, int32_t max_seqlen_kv, int32_t num_heads_q,
                            int32_t num_heads_kv, int32_t head_dim, int32_t cmp_topk, int32_t cmp_ratio,
                            int32_t ori_mask_mode, int32_t ori_win_left, int32_t layout_q, int32_t layout_kv,
                            int32_t has_cmp_kv, int32_t aic_core_num, int32_t* metadata_out, int32_t* status,
                            void* workspace, size_t workspace_bytes, void* stream, bool support_fd, int32_t aiv_core_num) {
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
  A.scan_cap = g_scan_cap;
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
  A.fast = (ori_mask_mode == 4 && ori_win_left >= 0 && ori_win_left < (1 << 30) && A.is_s1g && A.att_mode == 1 &&
            (!A.has_cmp || (cmp_ratio > 0 && cmp_topk >= 0)));
  const size_t need = sas_metadata_workspace_bytes((int32_t)(B > 0 ? B : 1), aic_core_num);
  if (!workspace || workspace_bytes < need) return SAS_ERR_WORKSPACE;
  const size_t b1 = (size_t)(B > 0 ? B : 1);
  long long* arrays = static_cast<long long*>(workspace);
  int64_t* core_out = reinterpret_cast<int64_t*>(static_cast<char*>(workspace) +
                                                 align_up(sizeof(long long) * (kNumArrays * b1 + 1), 256));
  // dynamic shared memory: the batch arrays plus a row-cost cache sized from
  // max_seqlen_q (the kernel skips the cache when the real rows do not fit),
  // so a decode batch does not ask for the whole carve-out
  size_t smem = kSmemCap;
  if (max_seqlen_q > 0) {
    const size_t arr = B <= kSmemBatches ? sizeof(long long) * (kNumArrays * b1 + 1) + 16 : 0;
    const size_t rows = max_seqlen_q > kSmallRows ? b1 * (((size_t)max_seqlen_q + 31) / 32) * 32 : 0;
    smem = std::min((size_t)kSmemCap, align_up(arr + rows * sizeof(int2) + rows / 32 * sizeof(long long), 1024));
  }
  A.smem = (int)smem;
  if (smem > 48 * 1024) {
    int dev = 0;
    cudaGetDevice(&dev);
    static uint64_t attr_done = 0;
    if (!(attr_done & (1ull << (dev & 63)))) {
      if (cudaFuncSetAttribute(sas_metadata_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kSmemCap) != cudaSuccess)
        return SAS_ERR_CUDA;
      attr_done |= 1ull << (dev & 63);
    }
  }
  if (support_fd) {
    sas_metadata_fd_kernel<<<1, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(A, aiv_core_num, arrays, core_out,
                                                                                 metadata_out, status);
  } else {
    sas_metadata_kernel<<<1, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(A, arrays, core_out,
                                                                                  metadata_out, status);
  }
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}
}  // namespace

extern "C" int sas_metadata(const int32_t* cu_seqlens_q, int32_t n_cu_seqlens_q, const int32_t* cu_seqlens_ori_kv,
                            int32_t n_cu_seqlens_ori_kv, const int32_t* seqused_q, int32_t n_seqused_q,
                            const int32_t* seqused_kv, int32_t n_seqused_kv, int32_t batch_size,
                            int32_t max_seqlen_q, int32_t max_seqlen_kv, int32_t num_heads_q,
                            int32_t num_heads_kv, int32_t head_dim, int32_t cmp_topk, int32_t cmp_ratio,
                            int32_t ori_mask_mode, int32_t ori_win_left, int32_t layout_q, int32_t layout_kv,
                            int32_t has_cmp_kv, int32_t aic_core_num, int32_t* metadata_out, int32_t* status,
                            void* workspace, size_t workspace_bytes, void* stream) {
  return metadata_launch(cu_seqlens_q, n_cu_seqlens_q, cu_seqlens_ori_kv, n_cu_seqlens_ori_kv, seqused_q, n_seqused_q,
                         seqused_kv, n_seqused_kv, batch_size, max_seqlen_q, max_seqlen_kv, num_heads_q, num_heads_kv,
                         head_dim, cmp_topk, cmp_ratio, ori_mask_mode, ori_win_left, layout_q, layout_kv, has_cmp_kv,
                         aic_core_num, metadata_out, status, workspace, workspace_bytes, stream, false, 0);
}

extern "C" int sas_metadata_fd(const int32_t* cu_seqlens_q, int32_t n_cu_seqlens_q,
                               const int32_t* cu_seqlens_ori_kv, int32_t n_cu_seqlens_ori_kv,
                               const int32_t* seqused_q, int32_t n_seqused_q, const int32_t* seqused_kv,
                               int32_t n_seqused_kv, int32_t batch_size, int32_t max_seqlen_q, int32_t max_seqlen_kv,
                               int32_t num_heads_q, int32_t num_heads_kv, int32_t head_dim, int32_t cmp_topk,
                               int32_t cmp_ratio, int32_t ori_mask_mode, int32_t ori_win_left, int32_t layout_q,
                               int32_t layout_kv, int32_t has_cmp_kv, int32_t aic_core_num, int32_t aiv_core_num,
                               int32_t* metadata_out, int32_t* status, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (aiv_core_num < 0 || aiv_core_num > 72 + 64 || aic_core_num > SAS_AIC_CORE_NUM + 64) return SAS_ERR_INVALID_ARG;
  return metadata_launch(cu_seqlens_q, n_cu_seqlens_q, cu_seqlens_ori_kv, n_cu_seqlens_ori_kv, seqused_q, n_seqused_q,
                         seqused_kv, n_seqused_kv, batch_size, max_seqlen_q, max_seqlen_kv, num_heads_q, num_heads_kv,
                         head_dim, cmp_topk, cmp_ratio, ori_mask_mode, ori_win_left, layout_q, layout_kv, has_cmp_kv,
                         aic_core_num, metadata_out, status, workspace, workspace_bytes, stream, true, aiv_core_num);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of sas_metadata.
//
// Some callers cannot call cudaMalloc at the point where they need the
// schedule: code running while a caching allocator is locked or being
// torn down, plugins loaded into a host that owns all device memory, and
// hot loops that must not synchronise (cudaMalloc/cudaFree can). For them
// the scratch lives in a fixed device array compiled into this library.
// It is sized for up to kNoAllocMaxBatch requests and kNoAllocMaxCores
// cores (296,704 bytes), and every GPU that loads the library keeps that
// array until the process exits.
namespace {
constexpr int kNoAllocMaxBatch = 4096;
constexpr int kNoAllocMaxCores = 64;
constexpr size_t kNoAllocScratchBytes =
    ((sizeof(long long) * (kNumArrays * (size_t)kNoAllocMaxBatch + 1) + 255) / 256) * 256 +
    ((sizeof(int64_t) * 3 * (size_t)kNoAllocMaxCores + 255) / 256) * 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
constexpr int kMaxDevices = 64;
void* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;
}  // namespace

extern "C" int sas_metadata_noalloc(const int32_t* cu_seqlens_q, int32_t n_cu_seqlens_q,
                                    const int32_t* cu_seqlens_ori_kv, int32_t n_cu_seqlens_ori_kv,
                                    const int32_t* seqused_q, int32_t n_seqused_q, const int32_t* seqused_kv,
                                    int32_t n_seqused_kv, int32_t batch_size, int32_t max_seqlen_q,
                                    int32_t max_seqlen_kv, int32_t num_heads_q, int32_t num_heads_kv,
                                    int32_t head_dim, int32_t cmp_topk, int32_t cmp_ratio, int32_t ori_mask_mode,
                                    int32_t ori_win_left, int32_t layout_q, int32_t layout_kv, int32_t has_cmp_kv,
                                    int32_t aic_core_num, int32_t* metadata_out, int32_t* status, void* stream) {
  if (!metadata_out) return SAS_ERR_INVALID_ARG;
  // the batch size exactly as sas_metadata resolves it (metadata.py:345-350)
  int64_t B = batch_size;
  if (n_seqused_q > 0 && seqused_q) B = n_seqused_q;
  else if (layout_q == SAS_LAYOUT_TND && n_cu_seqlens_q > 0 && cu_seqlens_q) B = n_cu_seqlens_q - 1;
  if (B > kNoAllocMaxBatch || aic_core_num > kNoAllocMaxCores) return SAS_ERR_NOALLOC_LIMIT;
  if (!sas::select_device_of(metadata_out)) return SAS_ERR_INVALID_ARG;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SAS_ERR_CUDA;
  void* scratch = nullptr;
  {
    // first call on a device: look up the device address of the array (the
    // host-side symbol is only a stand-in and must never reach a kernel)
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return SAS_ERR_CUDA;
      }
      g_noalloc_ptr[dev] = p;
    }
    scratch = g_noalloc_ptr[dev];
  }
  // every byte of scratch the kernel reads it has written earlier in the same
  // launch, so nothing needs clearing between calls
  return sas_metadata(cu_seqlens_q, n_cu_seqlens_q, cu_seqlens_ori_kv, n_cu_seqlens_ori_kv, seqused_q, n_seqused_q,
                      seqused_kv, n_seqused_kv, batch_size, max_seqlen_q, max_seqlen_kv, num_heads_q, num_heads_kv,
                      head_dim, cmp_topk, cmp_ratio, ori_mask_mode, ori_win_left, layout_q, layout_kv, has_cmp_kv,
                      aic_core_num, metadata_out, status, scratch, kNoAllocScratchBytes, stream);
}
