/*
 * TEST INFRASTRUCTURE ONLY -- CPU restatement of the SparseAttnSharedkv
 * metadata scheduler, used as the bit-exact checker for the GPU metadata
 * kernel. Nothing in the product path links or calls this file; only the
 * tests, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it.
 *
 * Restates sparse_attn_sharedkv_tilelang/metadata.py (the Python port of the
 * AICPU scheduler) step by step:
 *   params init           metadata.py:359-389
 *   s2 token range        metadata.py:479-501
 *   block range / tails   metadata.py:512-547
 *   cost table            metadata.py:428-477
 *   win / cmp s1g caches  metadata.py:549-621, gather 623-632, s1g 634-667
 *   split info / costs    metadata.py:671-714
 *   assign by batch/row   metadata.py:718-764
 *   flash-decode path     metadata.py:766-870, 925-954 (only with support_fd,
 *                         which the reference's scheduler leaves False,
 *                         metadata.py:323-325): assign by block 777-794,
 *                         FD records 796-827, cursor / force assign 829-870,
 *                         FD vector split 925-954
 *   per-core plan         metadata.py:872-923, schedule 956-972
 *   packing               metadata.py:974-1009
 * Python integers are unbounded; the few quantities that can exceed int64
 * (pre-token INT64_MAX plus a length difference) are carried in __int128.
 * Parity is pinned by tests/golden/metadata_cases.npz, produced by running
 * the reference metadata.py itself (tests/golden/make_golden.py).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define AIC_CORE_NUM 36
#define AIV_CORE_NUM 72
#define SAS_META_SIZE 1024
#define FA_METADATA_SIZE 8

#define WIN_NORMAL 0
#define WIN_TAIL 1
#define CMP_NORMAL 2
#define CMP_TAIL 3

#define INT64_MAX_V ((int64_t)0x7fffffffffffffffLL)
#define ROW_SCAN_CAP (1LL << 26)

typedef __int128 i128;

static int64_t fdiv(int64_t a, int64_t b) { /* Python floor division */
  int64_t q = a / b, r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) q -= 1;
  return q;
}
static int64_t fmod_py(int64_t a, int64_t b) { return a - fdiv(a, b) * b; }
static int64_t clip64(int64_t v, int64_t lo, int64_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

typedef struct {
  int64_t nq, nkv, hd;
  const int64_t *cu_q; int64_t n_cu_q;
  const int64_t *cu_kv; int64_t n_cu_kv;
  const int64_t *sq; int64_t n_sq;
  const int64_t *skv; int64_t n_skv;
  int64_t batch, max_q, max_kv, cmp_topk, cmp_ratio, mask_mode, win_left;
  int64_t layout_q; /* 0 BSND, 1 TND, 2 BSH, 3 other */
  int64_t layout_kv; /* 0 PA_ND, 1 TND */
  int64_t has_cmp;
  int64_t aic, aiv, support_fd;
  /* derived */
  int64_t pre_token, next_token, group, m_base, s2_base;
  int is_s1g, is_cfa, is_scfa, attention_mode;
  int64_t tc[4][4];
  int err;
} Sched;

typedef struct { int64_t b, s1, s2; i128 pre_lu, next_lu; } BatchC;
typedef struct {
  int64_t b, s1g, s2_start, s2_end, win_s2_start, win_s2_end, cmp_s2_start, cmp_s2_end;
  int64_t s1g_cost, s1g_lbc, s1g_block, s1g_nbc;
  int64_t win_block, win_cost, win_lbc, win_nbc;
  int64_t cmp_block, cmp_cost, cmp_lbc, cmp_nbc;
  int64_t cmp_tail, win_tail;
} S1GC;

typedef struct {
  int64_t *s1g_base_num, *s2_base_num, *s1g_tail, *s2_tail;
  int all_zero;
  int64_t *bn2_cost, *bn2_block, *bn2_lbc;
  int64_t total_block, total_cost, max_s1g_cost;
} Ctx;

static int64_t s1_size(Sched *S, int64_t b) {
  if (S->n_sq > 0) { if (b >= S->n_sq) { S->err = 3; return 0; } return S->sq[b]; }
  if (S->layout_q == 1 && S->n_cu_q > 0) {
    if (b + 1 >= S->n_cu_q) { S->err = 3; return 0; }
    return S->cu_q[b + 1] - S->cu_q[b];
  }
  return S->max_q;
}
static int64_t s2_size(Sched *S, int64_t b) {
  if (S->n_skv > 0) { if (b >= S->n_skv) { S->err = 3; return 0; } return S->skv[b]; }
  if (S->layout_kv == 1 && S->n_cu_kv > 0) {
    if (b + 1 >= S->n_cu_kv) { S->err = 3; return 0; }
    return S->cu_kv[b + 1] - S->cu_kv[b];
  }
  return S->max_kv;
}

static void params_init(Sched *S) {
  if (S->n_sq > 0) S->batch = S->n_sq;
  else if (S->layout_q == 1 && S->n_cu_q > 0) S->batch = S->n_cu_q - 1;
  if (S->mask_mode == 0) { S->pre_token = INT64_MAX_V; S->next_token = INT64_MAX_V; S->attention_mode = 0; }
  else if (S->mask_mode == 3) { S->pre_token = INT64_MAX_V; S->next_token = 0; S->attention_mode = 1; }
  else { S->pre_token = S->win_left > -1 ? S->win_left : INT64_MAX_V; S->next_token = 0; S->attention_mode = 1; }
  S->is_s1g = (S->layout_q == 0 || S->layout_q == 1 || S->layout_q == 2);
  S->group = S->nkv == 0 ? 0 : fdiv(S->nq, S->nkv);
  S->is_cfa = S->is_scfa = 0;
  if (S->has_cmp) { if (S->cmp_topk > 0) S->is_scfa = 1; else S->is_cfa = 1; }
  S->m_base = S->group;
  S->s2_base = 512;
}

static int64_t calc_cost(int64_t m, int64_t s2) { return 6 * ((m + 15) >> 4) + 10 * ((s2 + 63) >> 6); }

static void cost_table(Sched *S, int64_t s1n, int64_t s2n, int64_t s1t, int64_t wt, int64_t ct) {
  S->tc[WIN_NORMAL][WIN_NORMAL] = calc_cost(s1n, s2n);
  S->tc[WIN_TAIL][WIN_NORMAL] = s1t == 0 ? 0 : calc_cost(s1t, s2n);
  S->tc[WIN_NORMAL][WIN_TAIL] = wt == 0 ? 0 : calc_cost(s1n, wt);
  S->tc[WIN_TAIL][WIN_TAIL] = (s1t == 0 || wt == 0) ? 0 : calc_cost(s1t, wt);
  if (S->has_cmp) {
    S->tc[CMP_NORMAL][CMP_NORMAL] = calc_cost(s1n, s2n);
    S->tc[CMP_TAIL][CMP_NORMAL] = s1t == 0 ? 0 : calc_cost(s1t, s2n);
    S->tc[CMP_NORMAL][CMP_TAIL] = ct == 0 ? 0 : calc_cost(s1n, ct);
    S->tc[CMP_TAIL][CMP_TAIL] = (s1t == 0 || ct == 0) ? 0 : calc_cost(s1t, ct);
  }
}

static void batch_cache(Sched *S, int64_t b, BatchC *bc) {
  bc->b = b;
  bc->s1 = s1_size(S, b);
  bc->s2 = s2_size(S, b);
  bc->pre_lu = (S->mask_mode == 4) ? (i128)bc->s1 - bc->s2 + S->pre_token : (i128)S->pre_token;
  int64_t m = S->mask_mode;
  if (m == 0 || m == 1 || m == 2) bc->next_lu = S->next_token;
  else if (m == 3) bc->next_lu = (i128)bc->s2 - bc->s1;
  else if (m == 4) bc->next_lu = (i128)bc->s2 - bc->s1 + S->next_token;
  else bc->next_lu = S->next_token;
}

static void s2_token_range(Sched *S, int64_t s1g, BatchC *bc, i128 *first, i128 *last) {
  if (bc->s1 == 0 || bc->s2 == 0) { *first = 0; *last = 0; return; }
  if (!S->attention_mode) { *first = 0; *last = bc->s2 - 1; return; }
  int64_t g_first = s1g * S->m_base;
  int64_t lim = bc->s1 * S->group;
  int64_t g_last = (g_first + S->m_base < lim ? g_first + S->m_base : lim) - 1;
  int64_t f, l;
  if (S->is_s1g) { f = fdiv(g_first, S->group); l = fdiv(g_last, S->group); }
  else {
    if (fdiv(g_first, bc->s1) == fdiv(g_last, bc->s1)) { f = fmod_py(g_first, bc->s1); l = fmod_py(g_last, bc->s1); }
    else { f = 0; l = bc->s1; }
  }
  *first = (i128)f - bc->pre_lu;
  *last = (i128)l + bc->next_lu;
}

static void block_range(Sched *S, i128 f, i128 l, BatchC *bc, S1GC *sc) {
  int64_t of, ol;
  if (f >= bc->s2 || l < 0 || l < f) {
    of = 0; ol = 0; sc->win_s2_start = 0; sc->win_s2_end = 0; sc->win_tail = 0;
  } else {
    of = (int64_t)(f < 0 ? 0 : (f > bc->s2 - 1 ? bc->s2 - 1 : f));
    ol = (int64_t)(l < 0 ? 0 : (l > bc->s2 - 1 ? bc->s2 - 1 : l));
    sc->win_s2_start = 0;
    sc->win_s2_end = fdiv(ol - of, S->s2_base) + 1;
    sc->win_tail = fmod_py(ol - of + 1, S->s2_base);
  }
  (void)of;
  sc->cmp_s2_start = sc->win_s2_end;
  int64_t last_tok = (S->has_cmp && S->cmp_ratio > 0) ? fdiv(ol + 1, S->cmp_ratio) : 0;
  int64_t act = 0;
  if (S->is_cfa) act = last_tok;
  else if (S->is_scfa) act = last_tok < S->cmp_topk ? last_tok : S->cmp_topk;
  if (act == 0) sc->cmp_s2_end = sc->cmp_s2_start;
  else sc->cmp_s2_end = sc->cmp_s2_start + fdiv(act - 1, S->s2_base) + 1;
  sc->cmp_tail = fmod_py(act, S->s2_base);
}

static void win_cache(Sched *S, S1GC *sc, Ctx *C) {
  if (sc->win_s2_start >= sc->win_s2_end) { sc->win_block = sc->win_cost = sc->win_lbc = sc->win_nbc = 0; return; }
  sc->win_block = sc->win_s2_end - sc->win_s2_start;
  int64_t t = sc->win_tail != 0 ? 1 : 0, n = sc->win_block - t;
  if (sc->s1g == C->s1g_base_num[sc->b] - 1 && C->s1g_tail[sc->b] != 0) {
    sc->win_cost = S->tc[WIN_TAIL][WIN_NORMAL] * n + S->tc[WIN_TAIL][WIN_TAIL] * t;
    sc->win_lbc = t > 0 ? S->tc[WIN_TAIL][WIN_TAIL] : S->tc[WIN_TAIL][WIN_NORMAL];
    sc->win_nbc = S->tc[WIN_TAIL][WIN_NORMAL];
  } else {
    sc->win_cost = S->tc[WIN_NORMAL][WIN_NORMAL] * n + S->tc[WIN_NORMAL][WIN_TAIL] * t;
    sc->win_lbc = t > 0 ? S->tc[WIN_NORMAL][WIN_TAIL] : S->tc[WIN_NORMAL][WIN_NORMAL];
    sc->win_nbc = S->tc[WIN_NORMAL][WIN_NORMAL];
  }
}

static void cmp_cache(Sched *S, S1GC *sc, Ctx *C) {
  if (sc->cmp_s2_start >= sc->cmp_s2_end) { sc->cmp_block = sc->cmp_cost = sc->cmp_lbc = sc->cmp_nbc = 0; return; }
  sc->cmp_block = sc->cmp_s2_end - sc->cmp_s2_start;
  int64_t t = sc->cmp_tail != 0 ? 1 : 0, n = sc->cmp_block - t;
  if (sc->s1g == C->s1g_base_num[sc->b] - 1 && C->s1g_tail[sc->b] != 0) {
    sc->cmp_cost = S->tc[CMP_TAIL][CMP_NORMAL] * n + S->tc[CMP_TAIL][CMP_TAIL] * t;
    sc->cmp_lbc = t > 0 ? S->tc[CMP_TAIL][CMP_TAIL] : S->tc[CMP_TAIL][CMP_NORMAL];
    sc->cmp_nbc = S->tc[CMP_TAIL][CMP_NORMAL];
  } else {
    sc->cmp_cost = S->tc[CMP_NORMAL][CMP_NORMAL] * n + S->tc[CMP_NORMAL][CMP_TAIL] * t;
    sc->cmp_lbc = t > 0 ? S->tc[CMP_NORMAL][CMP_TAIL] : S->tc[CMP_NORMAL][CMP_NORMAL];
    sc->cmp_nbc = S->tc[CMP_NORMAL][CMP_NORMAL];
  }
}

static void s1g_cache(Sched *S, int64_t s1g, Ctx *C, BatchC *bc, S1GC *sc) {
  if (C->s1g_base_num[bc->b] == 0) {
    sc->s1g_cost = 0; sc->s1g_lbc = 0; sc->win_nbc = 0; sc->win_lbc = 0; sc->cmp_nbc = 0; sc->cmp_lbc = 0;
    sc->s1g_block = 0; sc->s2_start = 0; sc->cmp_s2_start = 0; sc->s2_end = 0;
    return;
  }
  sc->b = bc->b;
  sc->s1g = s1g;
  i128 f, l;
  s2_token_range(S, s1g, bc, &f, &l);
  block_range(S, f, l, bc, sc);
  cost_table(S, S->m_base, S->s2_base, C->s1g_tail[sc->b], sc->win_tail, sc->cmp_tail);
  win_cache(S, sc, C);
  cmp_cache(S, sc, C);
  sc->s2_start = sc->win_block > 0 ? sc->win_s2_start : sc->cmp_s2_start;
  if (sc->cmp_block > 0) { sc->s1g_lbc = sc->cmp_lbc; sc->s2_end = sc->cmp_s2_end; }
  else { sc->s1g_lbc = sc->win_lbc; sc->s2_end = sc->win_s2_end; }
  sc->s1g_block = sc->win_block + sc->cmp_block;
  sc->s1g_cost = sc->win_cost + sc->cmp_cost;
}

typedef struct {
  int64_t cur_b, cur_bn2, cur_s1g, cur_s2, cur_core, unassigned, bn2_cost, bn2_block;
  int64_t kv_split_part, fd_data_num;
  int finished;
  BatchC bc;
  S1GC sc;
  int64_t core_limit, core_cost, core_block;
} Assign;

static void assign_by_batch(Sched *S, Ctx *C, Assign *A) {
  if (A->finished) return;
  while (A->bn2_cost == 0 || A->core_limit + fdiv(C->bn2_lbc[A->cur_b], 2) >= A->core_cost + A->bn2_cost) {
    A->core_cost += A->bn2_cost;
    A->core_block += A->bn2_block;
    A->cur_bn2 += 1;
    if (A->cur_bn2 == S->batch * S->nkv) { A->cur_s1g = 0; A->cur_s2 = 0; A->finished = 1; return; }
    if (fdiv(A->cur_bn2, S->nkv) != A->cur_b) { A->cur_b = fdiv(A->cur_bn2, S->nkv); batch_cache(S, A->cur_b, &A->bc); }
    A->bn2_cost = C->bn2_cost[A->cur_b];
    A->bn2_block = C->bn2_block[A->cur_b];
    A->cur_s1g = 0;
    s1g_cache(S, A->cur_s1g, C, &A->bc, &A->sc);
    A->cur_s2 = A->sc.s2_start;
    if (S->err) return;
  }
}

static void assign_by_row(Sched *S, Ctx *C, Assign *A) {
  if (A->finished) return;
  int64_t guard = 0;
  while (A->core_limit + fdiv(A->sc.s1g_lbc, 2) >= A->core_cost + A->sc.s1g_cost) {
    A->core_cost += A->sc.s1g_cost;
    A->core_block += A->sc.s1g_block;
    A->bn2_cost = A->bn2_cost - A->sc.s1g_cost; if (A->bn2_cost < 0) A->bn2_cost = 0;
    A->bn2_block = A->bn2_block - A->sc.s1g_block; if (A->bn2_block < 0) A->bn2_block = 0;
    for (;;) {
      A->cur_s1g += 1;
      s1g_cache(S, A->cur_s1g, C, &A->bc, &A->sc);
      if (A->sc.s1g_block != 0) break;
      if (++guard > ROW_SCAN_CAP) { S->err = 2; return; }
    }
    A->cur_s2 = A->sc.s2_start;
    if (++guard > ROW_SCAN_CAP) { S->err = 2; return; }
  }
}

/* ---- flash-decode path (support_fd) ---- */
static int64_t cur_block_cost(Assign *A) { /* metadata.py:766-775 */
  if (A->cur_s2 < A->sc.cmp_s2_start) {
    return A->cur_s2 == A->sc.cmp_s2_start - 1 ? A->sc.win_lbc : A->sc.win_nbc;
  }
  return A->cur_s2 == A->sc.s2_end - 1 ? A->sc.cmp_lbc : A->sc.cmp_nbc;
}

static void assign_by_block(Assign *A) { /* metadata.py:777-794 */
  if (A->finished) return;
  int64_t c = cur_block_cost(A);
  int64_t guard = 0;
  while (A->core_limit + fdiv(c, 2) >= A->core_cost + c) {
    A->core_cost += c;
    A->core_block += 1;
    A->cur_s2 += 1;
    A->bn2_cost -= c;
    A->sc.s1g_cost -= c;
    A->bn2_block -= 1;
    A->sc.s1g_block -= 1;
    c = cur_block_cost(A);
    if (++guard > ROW_SCAN_CAP) return;
  }
}

static void update_cursor(Sched *S, Ctx *C, Assign *A) { /* metadata.py:829-857 */
  int upd_s1g = 0, upd_b = 0;
  if (A->cur_s2 >= A->sc.s2_end) { A->cur_s2 = 0; A->cur_s1g += 1; upd_s1g = 1; }
  if (A->cur_s1g >= C->s1g_base_num[A->cur_b]) { A->cur_s1g = 0; A->cur_bn2 += 1; }
  if (A->cur_bn2 == S->batch * S->nkv) { A->cur_s1g = 0; A->cur_s2 = 0; A->finished = 1; return; }
  if (fdiv(A->cur_bn2, S->nkv) != A->cur_b) { A->cur_b = fdiv(A->cur_bn2, S->nkv); A->cur_s1g = 0; upd_b = 1; upd_s1g = 1; }
  if (upd_b) { batch_cache(S, A->cur_b, &A->bc); A->bn2_cost = C->bn2_cost[A->cur_b]; A->bn2_block = C->bn2_block[A->cur_b]; }
  if (upd_s1g) { s1g_cache(S, A->cur_s1g, C, &A->bc, &A->sc); A->cur_s2 = A->sc.win_s2_start; }
}

static void force_assign(Sched *S, Ctx *C, Assign *A) { /* metadata.py:859-870 */
  if (A->finished) return;
  int64_t c = cur_block_cost(A);
  A->core_cost += c;
  A->core_block += 1;
  A->cur_s2 += 1;
  A->bn2_cost -= c;
  A->bn2_block -= 1;
  A->sc.s1g_cost -= c;
  A->sc.s1g_block -= 1;
  update_cursor(S, C, A);
}

typedef struct { /* FlashDecodeResult + the SplitResult FD fields, metadata.py:206-252 */
  int64_t n_head, max_split, used_vec;
  int64_t bn2[AIC_CORE_NUM + 64], m[AIC_CORE_NUM + 64], ws[AIC_CORE_NUM + 64], split[AIC_CORE_NUM + 64],
      msize[AIC_CORE_NUM + 64];
  int64_t idx[AIV_CORE_NUM + 64], m_start[AIV_CORE_NUM + 64], m_num[AIV_CORE_NUM + 64];
} FdRes;

static void record_fd(Sched *S, Ctx *C, Assign *A, const int64_t *bn2_end, const int64_t *g_s1_end,
                      FdRes *F) { /* metadata.py:807-827 */
  int64_t split_b = fdiv(bn2_end[A->cur_core - 1], S->nkv);
  int64_t split_s1g = g_s1_end[A->cur_core - 1];
  int64_t s1 = s1_size(S, split_b);
  int64_t msz = split_s1g == C->s1g_base_num[split_b] - 1 ? s1 * S->group - split_s1g * S->m_base : S->m_base;
  if (A->kv_split_part > F->max_split) F->max_split = A->kv_split_part;
  int64_t h = F->n_head;
  if (h >= S->aic) { S->err = 5; return; } /* the reference's lists hold aic entries */
  F->bn2[h] = bn2_end[A->cur_core - 1];
  F->m[h] = g_s1_end[A->cur_core - 1];
  F->ws[h] = A->fd_data_num - A->kv_split_part;
  F->split[h] = A->kv_split_part;
  F->msize[h] = msz;
  F->n_head += 1;
}

static void split_fd(Sched *S, FdRes *F) { /* metadata.py:925-954 */
  int64_t total = 0;
  for (int64_t i = 0; i < F->n_head; ++i) total += F->split[i] * F->msize[i];
  if (S->aiv == 0) return;
  int64_t avg = fdiv(total, S->aiv);
  if (avg == 0) return;
  int64_t cur = 0;
  for (int64_t i = 0; i < F->n_head; ++i) {
    int64_t nv = fdiv(F->split[i] * F->msize[i], avg);
    if (nv == 0) continue;
    int64_t ave = fdiv(F->msize[i], nv);
    for (int64_t v = 0; v < nv; ++v) {
      if (cur >= S->aiv) break; /* len(fd_idx) == aiv_core_num */
      F->idx[cur] = i;
      F->m_start[cur] = v * ave;
      F->m_num[cur] = v < nv - 1 ? ave : F->msize[i] - v * ave;
      cur += 1;
    }
  }
  F->used_vec = cur;
}

int sas_meta_oracle(int64_t nq, int64_t nkv, int64_t hd,
                    const int64_t *cu_q, int64_t n_cu_q,
                    const int64_t *cu_kv, int64_t n_cu_kv,
                    const int64_t *sq, int64_t n_sq,
                    const int64_t *skv, int64_t n_skv,
                    int64_t batch, int64_t max_q, int64_t max_kv,
                    int64_t cmp_topk, int64_t cmp_ratio, int64_t mask_mode, int64_t win_left,
                    int64_t layout_q, int64_t layout_kv, int64_t has_cmp, int64_t aic,
                    int64_t aiv, int64_t support_fd, int32_t *out) {
  Sched S;
  memset(&S, 0, sizeof(S));
  S.nq = nq; S.nkv = nkv; S.hd = hd;
  S.cu_q = cu_q; S.n_cu_q = n_cu_q; S.cu_kv = cu_kv; S.n_cu_kv = n_cu_kv;
  S.sq = sq; S.n_sq = n_sq; S.skv = skv; S.n_skv = n_skv;
  S.batch = batch; S.max_q = max_q; S.max_kv = max_kv;
  S.cmp_topk = cmp_topk; S.cmp_ratio = cmp_ratio; S.mask_mode = mask_mode; S.win_left = win_left;
  S.layout_q = layout_q; S.layout_kv = layout_kv; S.has_cmp = has_cmp; S.aic = aic;
  S.aiv = aiv; S.support_fd = support_fd;
  if (aic > AIC_CORE_NUM + 64 || aiv > AIV_CORE_NUM + 64) return 1;
  memset(out, 0, sizeof(int32_t) * SAS_META_SIZE);
  params_init(&S);
  if (S.batch < 0 || S.aic < 0 || S.nkv <= 0 || S.group <= 0) return 1;
  int64_t B = S.batch, NC = S.aic > 0 ? S.aic : 1;
  int64_t *mem = (int64_t *)calloc((size_t)(7 * (B + 1) + 3 * NC), sizeof(int64_t));
  if (!mem) return 4;
  Ctx C;
  memset(&C, 0, sizeof(C));
  C.s1g_base_num = mem; C.s2_base_num = mem + (B + 1); C.s1g_tail = mem + 2 * (B + 1); C.s2_tail = mem + 3 * (B + 1);
  C.bn2_cost = mem + 4 * (B + 1); C.bn2_block = mem + 5 * (B + 1); C.bn2_lbc = mem + 6 * (B + 1);
  int64_t *bn2_end = mem + 7 * (B + 1), *g_s1_end = bn2_end + NC, *s2_end = g_s1_end + NC;
  int64_t used = 0;
  FdRes F;
  memset(&F, 0, sizeof(F));

  /* _calc_split_info */
  C.all_zero = 1;
  for (int64_t b = 0; b < B; ++b) {
    int64_t s1 = s1_size(&S, b), s2 = s2_size(&S, b);
    C.s1g_base_num[b] = fdiv(s1 * S.group + S.m_base - 1, S.m_base);
    C.s1g_tail[b] = fmod_py(s1 * S.group, S.m_base);
    C.s2_base_num[b] = fdiv(s2 + S.s2_base - 1, S.s2_base);
    C.s2_tail[b] = fmod_py(s2, S.s2_base);
    if (C.s1g_base_num[b] != 0 && C.s2_base_num[b] != 0) C.all_zero = 0;
  }
  if (S.err) { free(mem); return S.err; }
  if (C.all_zero) {
    used = 1; bn2_end[0] = B * S.nkv; g_s1_end[0] = 0; s2_end[0] = 0;
  } else {
    /* _calc_cost_info */
    for (int64_t b = 0; b < B; ++b) {
      C.bn2_cost[b] = C.bn2_block[b] = C.bn2_lbc[b] = 0;
      if (s1_size(&S, b) == 0 || s2_size(&S, b) == 0) continue;
      BatchC bc; S1GC sc; memset(&bc, 0, sizeof(bc)); memset(&sc, 0, sizeof(sc));
      batch_cache(&S, b, &bc);
      for (int64_t g = 0; g < C.s1g_base_num[b]; ++g) {
        s1g_cache(&S, g, &C, &bc, &sc);
        C.bn2_cost[b] += sc.s1g_cost;
        C.bn2_block[b] += sc.s1g_block;
        if (sc.s1g_cost > C.max_s1g_cost) C.max_s1g_cost = sc.s1g_cost;
        if (sc.s1g_block > 0) C.bn2_lbc[b] = sc.s1g_lbc;
      }
      C.total_cost += C.bn2_cost[b] * S.nkv;
      C.total_block += C.bn2_block[b] * S.nkv;
    }
    /* _calc_split_plan */
    used = 1;
    if (S.aic != 0) {
      Assign A; memset(&A, 0, sizeof(A));
      A.kv_split_part = 1; A.fd_data_num = 1;
      int64_t max_cost = 0;
      A.unassigned = C.total_cost;
      A.bn2_cost = C.bn2_cost[0];
      A.bn2_block = C.bn2_block[0];
      batch_cache(&S, 0, &A.bc);
      s1g_cache(&S, 0, &C, &A.bc, &A.sc);
      A.cur_s2 = A.sc.s2_start;
      for (int64_t i = 0; i < S.aic; ++i) {
        if (A.finished || A.unassigned <= 0) break;
        A.cur_core = i;
        int64_t den = S.aic - A.cur_core; if (den < 1) den = 1;
        int64_t avg = fdiv(A.unassigned, den);
        A.core_cost = 0; A.core_block = 0;
        A.core_limit = S.support_fd ? avg : (avg > C.max_s1g_cost ? avg : C.max_s1g_cost);
        assign_by_batch(&S, &C, &A);
        if (S.err) break;
        assign_by_row(&S, &C, &A);
        if (S.err) break;
        if (S.support_fd) {
          assign_by_block(&A);
          if (A.core_block == 0) force_assign(&S, &C, &A);
          if (S.err) break;
        }
        bn2_end[A.cur_core] = A.cur_bn2;
        g_s1_end[A.cur_core] = A.cur_s1g;
        s2_end[A.cur_core] = A.cur_s2;
        if (A.core_cost > max_cost) max_cost = A.core_cost;
        A.unassigned -= A.core_cost;
        /* _is_need_record_fd (metadata.py:796-805) */
        if (A.cur_core != 0 && A.kv_split_part > 1 &&
            !(A.cur_bn2 == bn2_end[A.cur_core - 1] && A.cur_s1g == g_s1_end[A.cur_core - 1])) {
          record_fd(&S, &C, &A, bn2_end, g_s1_end, &F);
          if (S.err) break;
          A.kv_split_part = 1;
        }
        if (A.sc.s2_start < A.cur_s2 && A.cur_s2 <= A.sc.s2_end) A.kv_split_part += 1;
      }
      used = A.cur_core + 1;
    }
    if (F.n_head > 0) split_fd(&S, &F);
    if (used < 1) used = 1;
  }
  if (S.err) { free(mem); return S.err; }
  /* _gen_metadata (first_fd_data_workspace_idx is never assigned: 0) */
  for (int64_t i = 0; i < AIC_CORE_NUM; ++i) {
    int32_t *row = out + i * FA_METADATA_SIZE;
    if (i >= used || i >= S.aic) { row[0] = 0; continue; }
    row[0] = 1;
    row[1] = (int32_t)(i == 0 ? 0 : bn2_end[i - 1]);
    row[2] = (int32_t)(i == 0 ? 0 : g_s1_end[i - 1]);
    row[3] = (int32_t)(i == 0 ? 0 : s2_end[i - 1]);
    row[4] = (int32_t)bn2_end[i];
    row[5] = (int32_t)g_s1_end[i];
    row[6] = (int32_t)s2_end[i];
    row[7] = 0;
  }
  for (int64_t i = 0; i < AIV_CORE_NUM; ++i) {
    int32_t *row = out + AIC_CORE_NUM * FA_METADATA_SIZE + i * 8;
    if (i >= F.used_vec || i >= S.aiv) { row[0] = 0; continue; }
    int64_t f = F.idx[i];
    row[0] = 1;
    row[1] = (int32_t)F.bn2[f];
    row[2] = (int32_t)F.m[f];
    row[3] = (int32_t)F.ws[f];
    row[4] = (int32_t)F.split[f];
    row[5] = (int32_t)F.m_start[i];
    row[6] = (int32_t)F.m_num[i];
  }
  free(mem);
  return 0;
}
