// Cluster decode variant of the sparse shared-KV attention forward (sm_100a).
//
// The tiled kernel (sas_fwd.cu) runs each query token's tiles on one CTA, so
// the exact tile max forces two copies of every 128-row chunk into shared
// memory (scores first, P.V after the tile max), and a batch of few tokens
// leaves SMs idle. Here a cluster of four CTAs shares each (token, 64-head
// group) unit, golden.py's tiles spread over the cluster:
//   - the window tile (<= 128 rows, golden.py:120-150): 32 rows per CTA;
//   - compressed tile i (512 rows, golden.py:156-200): chunk 4i + rank on
//     CTA `rank`.
// Each CTA copies its rows into shared memory ONCE, computes S^T = K Q^T
// (tcgen05, TMEM), takes its rows' per-head max, and the four CTAs exchange
// max(local max, running max) through distributed shared memory: every CTA
// then holds the exact running max of golden.py after that tile, and rounds
// P at the same points. P.V runs on the same resident rows. At the end of a
// unit the four partial O (same running max on every CTA, so no rescale) are
// summed: CTA d owns output columns [128d, 128d+128) and reads the other three
// CTAs' partials of those columns through L2 (fixed order, deterministic);
// the row sums l travel through distributed shared memory.
//
// Warp roles (12 warps): 0-1 loaders (cp.async of the valid rows only), 2
// MMA issuer and TMEM owner, 3 row resolution (kernel.py:285-401, 686-766;
// golden.py:28-66 top-k scan) up to CD steps ahead, 4-11 softmax / epilogue
// in two groups of 32 heads. Every wait is bounded; remote arrivals use
// release / acquire at cluster scope.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "sas_common.cuh"

namespace {

constexpr int D = 512;
constexpr int HG = 64;
constexpr int CH = 128;
constexpr int NSLAB = 8;
constexpr int SLAB_BYTES = CH * 128;
constexpr int Q_SLAB_BYTES = HG * 128;
constexpr int CL = 4;          // CTAs per cluster
constexpr int WP = CH / CL;    // window rows per CTA
constexpr int kThreads = 384;
constexpr int kLoaderWarps = 2, kMmaWarp = 2, kCoordWarp = 3, kSoftmaxWarpB = 8;  // softmax: warps 4-11
constexpr int CD = 4;          // row-resolution ring depth, in steps
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

constexpr int OFF_Q = 0;
constexpr int OFF_KV = OFF_Q + NSLAB * Q_SLAB_BYTES;
constexpr int OFF_P = OFF_KV + NSLAB * SLAB_BYTES;
constexpr int OFF_MISC = OFF_P + CH * 128;
constexpr int M_BAR = 0;                    // 64 mbarriers
constexpr int M_TMEM = 512;
constexpr int M_CTL = 520;                  // sas::CtaCtl
constexpr int M_SWA = 544;                  // 3 OR words, softmax group A
constexpr int M_SWB = 560;                  // 3 OR words, softmax group B
constexpr int M_COORD = 576;                // [CD][128] pool row (-1 = masked)
constexpr int M_CMASK = M_COORD + CD * CH * 4;  // [CD][4] validity words
constexpr int M_CINFO = M_CMASK + CD * 16;      // [CD] int4 {flags, unit, step, 0}
constexpr int M_RED = M_CINFO + CD * 16;        // [4 quads][64] per-warp maxima / row sums
constexpr int M_MRUN = M_RED + 1024;            // [2 groups][4 quads][32] running max per warp
constexpr int M_X = M_MRUN + 1024;              // [2 parity][4 src][64] exchanged maxima
constexpr int M_L = M_X + 2048;                 // [2 parity][4 src][64] exchanged row sums
constexpr int M_LRED = M_L + 2048;              // [4 quads][64] per-warp row sums of a unit
constexpr int MISC_BYTES = M_LRED + 1024;
constexpr int SMEM_BYTES = OFF_MISC + MISC_BYTES + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory over the per-CTA limit");

constexpr int B_FULL = 0;      // NSLAB: slab filled (64 loader threads)
constexpr int B_EMPTY = 8;     // rows and P buffer free: P.V of the last filled step done
constexpr int B_QFULL = 9;
constexpr int B_QEMPTY = 10;
constexpr int B_SF = 11;       // S^T in TMEM
constexpr int B_PREADY = 12;   // softmax done with the step (256)
constexpr int B_OFULL = 13;    // the unit's O^T complete
constexpr int B_OEMPTY = 14;   // the epilogue has read O^T (256)
constexpr int B_CFULL = 15;    // CD
constexpr int B_CEMPTY = 19;   // CD
constexpr int B_XA = 23;       // 2 (parity): maxima from the 4 CTAs, group A (128 arrivals)
constexpr int B_XB = 25;       // 2
constexpr int B_REDA = 27;     // 2 (parity): partials from the 3 other CTAs, group A (384 arrivals)
constexpr int B_REDB = 29;     // 2
constexpr int B_SYNCA = 31;
constexpr int B_SYNCB = 32;
constexpr int B_DRAIN = 33;
constexpr int kCemptyCount = kLoaderWarps + 8 + 1;

enum : int {
  DF_END = 1,     // no more steps
  DF_FIRST = 2,   // first step of a unit
  DF_LAST = 4,    // last step of a unit
  DF_EMPTY = 8,   // no valid row on this CTA
  DF_DEAD = 16,   // the unit's token has no work (padding): zero output, no exchange
  DF_WIN = 32,    // rows from the raw (window) pool, else compressed
};

constexpr uint32_t TM_S = 0;
constexpr uint32_t TM_O = 256;

struct DecParams {
  int T, H, G, B, S, layout, scenario, K, ratio, win_left;
  int ori_bs, ori_bt_stride, cmp_bs, cmp_bt_stride, ori_nblk, cmp_nblk;
  const uint8_t* ori_kv;
  const uint8_t* cmp_kv;
  const int32_t* ori_bt;
  const int32_t* cmp_bt;
  const int32_t* idx;
  const int32_t* cu;
  const int32_t* seqused_kv;
  const int32_t* meta;
  const float* sinks;
  float scale_log2;
  void* out;
  float* lse;
  float* red_ws;  // [clusters][4 dst][4 src][2 groups][128 d][32 heads]
  int32_t* status;
  int q_box_h, early;
  unsigned long long wait_ns;
};

struct TokD {
  int b, s_g, thr, n_cmp, live;
};

__device__ __forceinline__ int py_floordiv(int a, int b) {
  int q = a / b, r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) --q;
  return q;
}

// Request and position of token t (api.py:208-240 layouts), one warp: the
// request is found with a 32-way search of cu_seqlens_q.
__device__ TokD token_info(const DecParams& p, int t, int lane) {
  int b, s, act_q;
  if (p.layout == SAS_LAYOUT_TND) {
    int lo = 0, hi = p.B - 1;  // last b with cu[b] <= t
    while (hi > lo) {
      const int step = (hi - lo + 32) / 32;
      const int probe = lo + (lane + 1) * step;
      const unsigned bal = __ballot_sync(0xffffffffu, probe <= hi && p.cu[probe] <= t);
      if (bal == 0) {
        hi = lo + step - 1;
      } else {
        const int k = 31 - __clz(bal);
        lo = lo + (k + 1) * step;
        hi = min(hi, lo + step - 1);
      }
    }
    b = lo;
    s = t - p.cu[b];
    act_q = p.cu[b + 1] - p.cu[b];
  } else {
    b = t / p.S;
    s = t - b * p.S;
    act_q = p.cu ? p.cu[b + 1] - p.cu[b] : p.S;
  }
  TokD k;
  k.b = b;
  k.live = b < p.B && s >= 0 && s < act_q;
  k.s_g = k.live ? p.seqused_kv[b] - act_q + s : -1;
  k.thr = max(py_floordiv(k.s_g + 1, p.ratio), 0);
  k.n_cmp = p.scenario == 3 ? min(p.K, k.thr) : (p.scenario == 2 ? k.thr : 0);
  return k;
}

__device__ __forceinline__ int unit_steps(const TokD& k) {
  if (!k.live) return 1;  // one dead step: zero output
  const int nch = (k.n_cmp + CH - 1) / CH;
  return 1 + (nch + CL - 1) / CL;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(sas::smem_u32(bar)) : "memory");
}

// Barrier among the 4 warps of a softmax group (bounded; OR-reduces pred).
struct GroupSync {
  uint64_t* bar;
  uint32_t* words;
  uint32_t ph;
  __device__ __forceinline__ bool sync_or(int pred, int lane, bool lead, int& result, volatile sas::CtaCtl* ctl,
                                          int* status, int where) {
    const bool any = __any_sync(0xffffffffu, pred);
    __syncwarp();
    const uint32_t k = ph % 3;
    if (lane == 0) {
      if (any) atomicOr(&words[k], 1u);
      if (lead) words[(k + 1) % 3] = 0;
      sas::mbar_arrive(bar);
    }
    const bool ok = sas::mbar_wait(bar, ph & 1, ctl, status, where);
    result = ok ? (int)*reinterpret_cast<volatile uint32_t*>(&words[k]) : 0;
    ++ph;
    return ok;
  }
  __device__ __forceinline__ bool sync(int lane, bool lead, volatile sas::CtaCtl* ctl, int* status, int where) {
    int unused;
    return sync_or(0, lane, lead, unused, ctl, status, where);
  }
};

template <int DT>
struct Io;
template <>
struct Io<0> {
  __device__ static uint32_t pack(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <>
struct Io<1> {
  __device__ static uint32_t pack(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

template <int DT>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(kThreads, 1)
    sas_dec_kernel(const __grid_constant__ CUtensorMap tm_q, const DecParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = sas::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  uint8_t* misc = smem + OFF_MISC;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + M_BAR);
  volatile sas::CtaCtl* ctl = reinterpret_cast<volatile sas::CtaCtl*>(misc + M_CTL);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + M_TMEM);
  int32_t* coords = reinterpret_cast<int32_t*>(misc + M_COORD);
  uint32_t* cmask = reinterpret_cast<uint32_t*>(misc + M_CMASK);
  int4* cinfo = reinterpret_cast<int4*>(misc + M_CINFO);
  float* red = reinterpret_cast<float*>(misc + M_RED);
  float* m_run = reinterpret_cast<float*>(misc + M_MRUN);
  float* xbuf = reinterpret_cast<float*>(misc + M_X);
  float* lbuf = reinterpret_cast<float*>(misc + M_L);
  float* lred = reinterpret_cast<float*>(misc + M_LRED);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = sas::cluster_ctarank();
  const int cl = (int)sas::cluster_id_x(), ncl = (int)sas::nclusters_x();
  const int U = p.T * p.G;

  if (tid == 0) {
    for (int i = 0; i < NSLAB; ++i) sas::mbar_init(&bars[B_FULL + i], 32 * kLoaderWarps);
    sas::mbar_init(&bars[B_EMPTY], 1);
    sas::mbar_init(&bars[B_QFULL], 1);
    sas::mbar_init(&bars[B_QEMPTY], 1);
    sas::mbar_init(&bars[B_SF], 1);
    sas::mbar_init(&bars[B_PREADY], 256);
    sas::mbar_init(&bars[B_OFULL], 1);
    sas::mbar_init(&bars[B_OEMPTY], 256);
    for (int i = 0; i < CD; ++i) {
      sas::mbar_init(&bars[B_CFULL + i], 1);
      sas::mbar_init(&bars[B_CEMPTY + i], kCemptyCount);
    }
    for (int i = 0; i < 2; ++i) {
      sas::mbar_init(&bars[B_XA + i], CL * 32);
      sas::mbar_init(&bars[B_XB + i], CL * 32);
      sas::mbar_init(&bars[B_REDA + i], (CL - 1) * 128);
      sas::mbar_init(&bars[B_REDB + i], (CL - 1) * 128);
    }
    sas::mbar_init(&bars[B_SYNCA], 4);
    sas::mbar_init(&bars[B_SYNCB], 4);
    sas::mbar_init(&bars[B_DRAIN], 1);
    for (int i = 0; i < 3; ++i) {
      reinterpret_cast<uint32_t*>(misc + M_SWA)[i] = 0;
      reinterpret_cast<uint32_t*>(misc + M_SWB)[i] = 0;
    }
    ctl->abort = 0;
    ctl->limit_ns = p.wait_ns;
    sas::fence_mbar_init();
  }
  // rows a step does not copy keep their old values; start from zeros so that
  // none of them can hold a non-finite pattern (masked rows get P = 0)
  for (int i = tid; i < (NSLAB * SLAB_BYTES + (p.q_box_h < HG ? NSLAB * Q_SLAB_BYTES : 0)) / 16; i += kThreads) {
    const int off = i * 16 < NSLAB * SLAB_BYTES ? OFF_KV + i * 16 : OFF_Q + (i * 16 - NSLAB * SLAB_BYTES);
    *reinterpret_cast<uint4*>(smem + off) = make_uint4(0, 0, 0, 0);
  }
  sas::fence_proxy_async_smem();
  if (warp == kMmaWarp) {
    sas::tmem_alloc(tmem_slot, 512);
    sas::tmem_relinquish();
  }
  if (!p.early) sas::pdl_wait();
  if (tid == 32) sas::tma_prefetch_desc(&tm_q);
  sas::tc_fence_before();
  __syncthreads();
  sas::cluster_sync();  // every CTA's barriers exist before any remote arrival
  sas::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kCoordWarp) {
    // =============================== row resolution, up to CD steps ahead
    uint32_t n = 0;
    bool ok = true;
    for (int u = cl; ok && u < U; u += ncl) {
      const int t = u / p.G;
      const TokD k = token_info(p, t, lane);
      const int steps = unit_steps(k);
      const int lo = max(k.s_g - p.win_left, 0);
      // first -1 among the top-k slots before the current chunk (golden.py:55-56)
      int scanned = 0;
      bool neg_before = false;
      for (int st = 0; ok && st < steps; ++st, ++n) {
        const int slot = n % CD;
        if (!sas::mbar_wait(&bars[B_CEMPTY + slot], ((n / CD) & 1) ^ 1, ctl, p.status, 2)) {
          ok = false;
          break;
        }
        int row[4];
        bool val[4];
        bool bad = false;
        const bool win = st == 0;
        if (!k.live) {
#pragma unroll
          for (int q = 0; q < 4; ++q) val[q] = false;
        } else if (win) {
          // window rows lo + 32*rank + lane (golden.py: [max(s_g-127,0), s_g])
#pragma unroll
          for (int q = 0; q < 4; ++q) val[q] = false;
          const int pos = lo + WP * (int)rank + lane;
          bool v = k.s_g >= 0 && pos <= k.s_g;
          const int col = pos / p.ori_bs;
          const bool in_table = col < p.ori_bt_stride;
          const int blk = v && in_table ? p.ori_bt[(size_t)k.b * p.ori_bt_stride + col] : -1;
          bad |= v && (!in_table || blk >= p.ori_nblk);
          val[0] = v && blk >= 0 && blk < p.ori_nblk;
          row[0] = blk * p.ori_bs + pos % p.ori_bs;
        } else {
          const int c = (st - 1) * CL + (int)rank;  // compressed chunk of this CTA
          const int e0 = c * CH;
          if (p.scenario == 3) {
            const int32_t* ip = p.idx + (size_t)t * p.K;
            const int lim = min(e0, k.n_cmp);
            int neg = 0;
            for (int e = scanned + lane; e < lim; e += 32) neg |= (ip[e] == -1);
            neg_before = neg_before || __any_sync(0xffffffffu, neg);
            scanned = max(scanned, lim);
            int id[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int e = e0 + q * 32 + lane;
              val[q] = e < k.n_cmp;
              id[q] = val[q] ? ip[e] : 0;
            }
            int cf = CH;  // first -1 in this chunk
#pragma unroll
            for (int q = 3; q >= 0; --q) {
              const unsigned bal = __ballot_sync(0xffffffffu, val[q] && id[q] == -1);
              if (bal) cf = q * 32 + __ffs(bal) - 1;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              val[q] = val[q] && !neg_before && q * 32 + lane < cf && id[q] >= 0 && id[q] < k.thr;
              row[q] = id[q];
            }
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int e = e0 + q * 32 + lane;
              val[q] = e < k.n_cmp && e < k.thr;
              row[q] = e;
            }
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int idv = row[q];
            const int col = idv / p.cmp_bs;
            const bool in_table = col < p.cmp_bt_stride;
            const int blk = val[q] && in_table ? p.cmp_bt[(size_t)k.b * p.cmp_bt_stride + col] : -1;
            bad |= val[q] && (!in_table || blk >= p.cmp_nblk);
            val[q] = val[q] && blk >= 0 && blk < p.cmp_nblk;
            row[q] = val[q] ? blk * p.cmp_bs + idv % p.cmp_bs : 0;
          }
        }
        if (__any_sync(0xffffffffu, bad) && lane == 0 && p.status) atomicCAS(p.status, 0, SAS_ERR_BAD_BLOCK_ENTRY);
        int any = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          coords[slot * CH + q * 32 + lane] = val[q] ? row[q] : -1;
          const unsigned vb = __ballot_sync(0xffffffffu, val[q]);
          any |= vb != 0;
          if (lane == 0) cmask[slot * 4 + q] = vb;
        }
        if (lane == 0) {
          const int fl = (st == 0 ? DF_FIRST : 0) | (st == steps - 1 ? DF_LAST : 0) | (any ? 0 : DF_EMPTY) |
                         (k.live ? 0 : DF_DEAD) | (win ? DF_WIN : 0);
          cinfo[slot] = make_int4(fl, u, st, 0);
        }
        __syncwarp();
        if (lane == 0) sas::mbar_arrive(&bars[B_CFULL + slot]);
      }
    }
    if (ok) {
      const int slot = n % CD;
      if (sas::mbar_wait(&bars[B_CEMPTY + slot], ((n / CD) & 1) ^ 1, ctl, p.status, 2) && lane == 0) {
        cinfo[slot] = make_int4(DF_END, 0, 0, 0);
        sas::mbar_arrive(&bars[B_CFULL + slot]);
      }
    }
  } else if (warp < kLoaderWarps) {
    // =============================== loaders: the step's valid rows, once
    const int lw = warp, sub = lane >> 3, c16 = lane & 7;
    const uint32_t kv_base = sas::smem_u32(smem + OFF_KV);
    const uint32_t q_bytes = (uint32_t)NSLAB * p.q_box_h * 128;
    uint32_t n = 0, fills = 0, qloads = 0;
    bool ok = true;
    while (ok) {
      const int slot = n % CD;
      if (!sas::mbar_wait(&bars[B_CFULL + slot], (n / CD) & 1, ctl, p.status, 3)) break;
      const int4 ci = cinfo[slot];
      if (ci.x & DF_END) break;
      if ((ci.x & DF_FIRST) && !(ci.x & DF_DEAD) && tid == 0) {
        if (!sas::mbar_wait(&bars[B_QEMPTY], (qloads & 1) ^ 1, ctl, p.status, 1)) {
          ok = false;
        } else {
          const int t = ci.y / p.G, g = ci.y % p.G;
          sas::mbar_arrive_expect_tx(&bars[B_QFULL], q_bytes);
          for (int s = 0; s < NSLAB; ++s)
            sas::tma_load_3d(smem + OFF_Q + s * Q_SLAB_BYTES, &tm_q, &bars[B_QFULL], s * 64, g * HG, t);
          ++qloads;
        }
      }
      if (ok && !(ci.x & DF_EMPTY)) {
        if (fills > 0 && !sas::mbar_wait(&bars[B_EMPTY], (fills - 1) & 1, ctl, p.status, 4)) {
          ok = false;
        } else {
          const uint8_t* pool = (ci.x & DF_WIN) ? p.ori_kv : p.cmp_kv;
          int crw[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) crw[i] = coords[slot * CH + lw * 64 + 4 * i + sub];
          for (int s = 0; s < NSLAB; ++s) {
            const uint32_t slab = kv_base + s * SLAB_BYTES;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int rl = lw * 64 + 4 * i + sub;
              if (crw[i] >= 0)
                cp_async16(slab + rl * 128 + ((c16 ^ (rl & 7)) << 4),
                           pool + (size_t)crw[i] * (D * 2) + s * 128 + c16 * 16);
            }
            cp_async_arrive(&bars[B_FULL + s]);
          }
          ++fills;
        }
      }
      __syncwarp();
      if (lane == 0) sas::mbar_arrive(&bars[B_CEMPTY + slot]);
      ++n;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (tid == 0 && qloads > 0) sas::mbar_wait_drain(&bars[B_QFULL], (qloads - 1) & 1, SAS_WAIT_LIMIT_NS);
  } else if (warp == kMmaWarp) {
    // =============================== MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc1 = sas::umma_idesc_f16(DT == 0 ? 1 : 0, 128, HG, 0, 0);
      constexpr uint32_t idesc2 = sas::umma_idesc_f16(DT == 0 ? 1 : 0, 128, HG, 1, 1);
      const uint32_t q_base = sas::smem_u32(smem + OFF_Q);
      const uint32_t kv_base = sas::smem_u32(smem + OFF_KV);
      const uint32_t p_base = sas::smem_u32(smem + OFF_P);
      uint32_t n = 0, fills = 0, qunits = 0, ounits = 0, o_writers = 0;
      int pv_in_unit = 0;
      bool ok = true;
      while (ok) {
        const int slot = n % CD;
        if (!sas::mbar_wait(&bars[B_CFULL + slot], (n / CD) & 1, ctl, p.status, 5)) break;
        const int4 ci = cinfo[slot];
        if (ci.x & DF_END) break;
        const bool empty = ci.x & DF_EMPTY;
        if (ci.x & DF_FIRST) {
          pv_in_unit = 0;
          if (!(ci.x & DF_DEAD)) {
            if (!sas::mbar_wait(&bars[B_QFULL], qunits & 1, ctl, p.status, 6)) break;
            ++qunits;
          }
        }
        if (!empty) {
          for (int s = 0; s < NSLAB && ok; ++s) {
            if (!sas::mbar_wait(&bars[B_FULL + s], fills & 1, ctl, p.status, 7)) {
              ok = false;
              break;
            }
            sas::fence_proxy_async_smem();
            sas::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sas::umma_desc_sw128(kv_base + s * SLAB_BYTES + kk * 32, 16, 1024);
              const uint64_t bd = sas::umma_desc_sw128(q_base + s * Q_SLAB_BYTES + kk * 32, 16, 1024);
              sas::umma_ss(tmem + TM_S, ad, bd, idesc1, (s | kk) != 0);
            }
          }
          if (!ok) break;
          sas::umma_commit(&bars[B_SF]);
        }
        if ((ci.x & DF_LAST) && !(ci.x & DF_DEAD)) sas::umma_commit(&bars[B_QEMPTY]);
        if (!sas::mbar_wait(&bars[B_PREADY], n & 1, ctl, p.status, 8)) break;
        if (!empty) {
          if (pv_in_unit == 0 && o_writers > 0 &&
              !sas::mbar_wait(&bars[B_OEMPTY], (ounits - 1) & 1, ctl, p.status, 9))
            break;
          sas::tc_fence_after();
          for (int j = 0; j < 4; ++j) {
            const uint32_t slot0 = kv_base + 2 * j * SLAB_BYTES;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t ad = sas::umma_desc_sw128(slot0 + kk * 2048, SLAB_BYTES, 1024);
              const uint64_t bd = sas::umma_desc_sw128(p_base + kk * 2048, 8192, 1024);
              sas::umma_ss(tmem + TM_O + 64 * j, ad, bd, idesc2, (pv_in_unit > 0 || kk > 0) ? 1u : 0u);
            }
          }
          sas::umma_commit(&bars[B_EMPTY]);
          ++pv_in_unit;
          ++fills;
        }
        if (ci.x & DF_LAST) {
          if (!(ci.x & DF_DEAD)) {
            sas::umma_commit(&bars[B_OFULL]);
            ++ounits;
            // the epilogue of every live unit arrives on B_OEMPTY once it has read O^T
            o_writers = 1;
          }
        }
        sas::mbar_arrive(&bars[B_CEMPTY + slot]);
        ++n;
      }
      sas::umma_commit(&bars[B_DRAIN]);
      sas::mbar_wait_drain(&bars[B_DRAIN], 0, SAS_WAIT_LIMIT_NS);
    }
    __syncwarp();
  } else {
    // =============================== softmax groups / epilogue
    const int quad = warp & 3;
    const int half = warp >= kSoftmaxWarpB ? 1 : 0;
    const int hb = 32 * half;
    const int gst = quad * 32 + lane;
    const bool lead = quad == 0;
    GroupSync gs{&bars[half ? B_SYNCB : B_SYNCA], reinterpret_cast<uint32_t*>(misc + (half ? M_SWB : M_SWA)), 0};
    const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
    float* mw = m_run + (half * 4 + quad) * 32;  // this warp's running max, heads hb..hb+31
    float lsum[32];
    uint32_t n = 0, sfills = 0, pvs = 0, xsteps = 0, ounits = 0, runits = 0;
    bool has_o = false, ok = true, waited_meta = false;
    const int xb = half ? B_XB : B_XA, rb = half ? B_REDB : B_REDA;
    while (ok) {
      const int slot = n % CD;
      if (!sas::mbar_wait(&bars[B_CFULL + slot], (n / CD) & 1, ctl, p.status, 10)) break;
      const int4 ci = cinfo[slot];
      if (ci.x & DF_END) break;
      const int u = ci.y, t = u / p.G, g = u % p.G;
      const bool empty = ci.x & DF_EMPTY, dead = ci.x & DF_DEAD;
      if (ci.x & DF_FIRST) {
        const int h = g * HG + hb + lane;
        mw[lane] = h < p.H ? p.sinks[h] * kLog2e : 0.f;  // (m, l) start at (sink, 1): golden.py:162-163
#pragma unroll
        for (int i = 0; i < 32; ++i) lsum[i] = 0.f;
        has_o = false;
      }
      __syncwarp();
      float al = 1.f;
      bool need = false;
      const bool valid = (cmask[slot * 4 + quad] >> lane) & 1;
      if (!dead) {
        // ---- this CTA's max over its rows of the tile, per head
        float tmx = -INFINITY;
        if (!empty) {
          if (!sas::mbar_wait(&bars[B_SF], sfills & 1, ctl, p.status, 11)) break;
          ++sfills;
          sas::tc_fence_after();
          uint32_t ra[32];
          sas::tmem_ld32(lane_addr + TM_S + hb, ra);
          sas::tmem_wait_ld();
          float mx[32];
#pragma unroll
          for (int h = 0; h < 32; ++h) mx[h] = valid ? __uint_as_float(ra[h]) * p.scale_log2 : -INFINITY;
#pragma unroll
          for (int h = 0; h < 32; h += 4) {
            float4 w;
            w.x = sas::warp_max_f32(mx[h]);
            w.y = sas::warp_max_f32(mx[h + 1]);
            w.z = sas::warp_max_f32(mx[h + 2]);
            w.w = sas::warp_max_f32(mx[h + 3]);
            if (lane == 0) *reinterpret_cast<float4*>(red + quad * 64 + hb + h) = w;
          }
          if (!gs.sync(lane, lead, ctl, p.status, 12)) break;
          tmx = fmaxf(fmaxf(red[hb + lane], red[64 + hb + lane]), fmaxf(red[128 + hb + lane], red[192 + hb + lane]));
        }
        // ---- exchange max(local max, running max) with the 4 CTAs of the cluster
        const uint32_t par = xsteps & 1;
        if (lead) {
          const float v = fmaxf(tmx, mw[lane]);
          const uint32_t xa = sas::smem_u32(xbuf + (par * CL + rank) * 64 + hb + lane);
          const uint32_t ba = sas::smem_u32(&bars[xb + par]);
#pragma unroll
          for (int q = 0; q < CL; ++q) sas::st_cluster_f32(sas::mapa_shared(xa, q), v);
#pragma unroll
          for (int q = 0; q < CL; ++q) sas::mbar_arrive_cluster(sas::mapa_shared(ba, q));
        }
        if (!sas::mbar_wait_cluster(&bars[xb + par], (xsteps >> 1) & 1, ctl, p.status, 13)) break;
        ++xsteps;
        {
          const float* xr = xbuf + par * CL * 64 + hb + lane;
          const float mn = fmaxf(fmaxf(xr[0], xr[64]), fmaxf(xr[128], xr[192]));
          const float mo = mw[lane];
          al = sas::ex2(mo - mn);
          need = __any_sync(0xffffffffu, mn > mo);
          __syncwarp();
          mw[lane] = mn;
          __syncwarp();
        }
        // ---- rescale l and O^T, then P = 2^(s - m) rounded into P^T
        if ((need && has_o) || !empty) {
          // O^T and the P buffer are free once the last P.V issued is done
          if (pvs > 0 && !sas::mbar_wait(&bars[B_EMPTY], (pvs - 1) & 1, ctl, p.status, 14)) break;
          sas::tc_fence_after();
        }
        if (need) {
#pragma unroll
          for (int h = 0; h < 32; ++h) lsum[h] *= __shfl_sync(0xffffffffu, al, h);
          if (has_o) {
#pragma unroll 1
            for (int j = 0; j < 4; ++j) {
              uint32_t o[32];
              sas::tmem_ld32(lane_addr + TM_O + 64 * j + hb, o);
              sas::tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < 32; ++h)
                o[h] = __float_as_uint(__uint_as_float(o[h]) * __shfl_sync(0xffffffffu, al, h));
              sas::tmem_st32(lane_addr + TM_O + 64 * j + hb, o);
            }
            sas::tmem_wait_st();
          }
        }
        if (!empty) {
          uint32_t ra[32];
          sas::tmem_ld32(lane_addr + TM_S + hb, ra);
          sas::tmem_wait_ld();
          float x[32];
#pragma unroll
          for (int h = 0; h < 32; ++h) x[h] = valid ? sas::ex2(__uint_as_float(ra[h]) * p.scale_log2 - mw[h]) : 0.f;
#pragma unroll
          for (int h = 0; h < 32; ++h) lsum[h] += x[h];
          uint8_t* prow = smem + OFF_P + gst * 128;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            const int cc = (hb >> 3) + c4;
            const int h = c4 * 8;
            *reinterpret_cast<uint4*>(prow + ((cc ^ (gst & 7)) << 4)) =
                make_uint4(Io<DT>::pack(x[h], x[h + 1]), Io<DT>::pack(x[h + 2], x[h + 3]),
                           Io<DT>::pack(x[h + 4], x[h + 5]), Io<DT>::pack(x[h + 6], x[h + 7]));
          }
          sas::fence_proxy_async_smem();
          ++pvs;
          has_o = true;
        }
      }
      sas::tc_fence_before();
      sas::mbar_arrive(&bars[B_PREADY]);
      __syncwarp();
      if (lane == 0) sas::mbar_arrive(&bars[B_CEMPTY + slot]);

      if (ci.x & DF_LAST) {
        // =========================== epilogue of the unit
        using T16 = uint16_t;
        T16* outp = reinterpret_cast<T16*>(p.out) + ((size_t)t * p.H + g * HG) * D;
        if (!waited_meta) {
          sas::pdl_wait();  // the metadata (and, in early mode, nothing else) is complete
          waited_meta = true;
        }
        // coverage by the metadata's core windows (kernel.py:254-278)
        int covered = 0;
        {
          const int tt = t;
          int b = 0, s = 0, smax = 0;
          // max_seq as the reference api computes it (api.py:208-215 / 229)
          if (p.layout == SAS_LAYOUT_TND) {
            for (int bb = lane; bb < p.B; bb += 32) smax = max(smax, p.cu[bb + 1] - p.cu[bb]);
            for (int o = 16; o; o >>= 1) smax = max(smax, __shfl_xor_sync(0xffffffffu, smax, o));
            int lo = 0, hi = p.B - 1;
            while (lo < hi) {
              const int mid = (lo + hi + 1) >> 1;
              if (p.cu[mid] <= tt) lo = mid;
              else hi = mid - 1;
            }
            b = lo;
            s = tt - p.cu[b];
          } else {
            smax = p.S;
            b = tt / p.S;
            s = tt - b * p.S;
          }
          const int pid = b * smax + s;
          int cov = 0;
          for (int c = lane; c < SAS_AIC_CORE_NUM; c += 32) {
            const int32_t* row = p.meta + c * 8;
            if (row[0] != 0 && pid >= row[1] * smax + row[2] && pid < row[4] * smax + row[5]) cov = 1;
          }
          covered = __any_sync(0xffffffffu, cov) && !dead;
        }
        const int d0 = (int)rank * 128;  // this CTA's output columns
        if (dead) {
          // padding: zero output and LSE (golden.py leaves them zero)
          for (int h = 0; h < 32; ++h) {
            const int hh = g * HG + hb + h;
            if (hh < p.H) outp[(size_t)(hb + h) * D + d0 + gst] = 0;
          }
          if (rank == 0 && lead && g * HG + hb + lane < p.H) p.lse[(size_t)t * p.H + g * HG + hb + lane] = 0.f;
        } else {
          // l over this CTA's rows, then to every CTA of the cluster
          float l[32];
#pragma unroll
          for (int h = 0; h < 32; ++h) l[h] = lsum[h];
#pragma unroll
          for (int step = 0; step < 5; ++step) {
            const int halfn = 16 >> step;
            const int m = 16 >> step;
            const bool up = (lane & m) != 0;
#pragma unroll
            for (int k2 = 0; k2 < halfn; ++k2) {
              const float a = l[k2], bb = l[k2 + halfn];
              const float send = up ? a : bb, keep = up ? bb : a;
              l[k2] = keep + __shfl_xor_sync(0xffffffffu, send, m);
            }
          }
          lred[quad * 64 + hb + lane] = l[0];
          if (!gs.sync(lane, lead, ctl, p.status, 15)) break;
          const uint32_t upar = runits & 1;
          // this CTA's l of head hb + lane (every warp of the group computes it)
          const float l_self = lred[hb + lane] + lred[64 + hb + lane] + lred[128 + hb + lane] + lred[192 + hb + lane];
          if (lead) {
            const uint32_t la = sas::smem_u32(lbuf + (upar * CL + rank) * 64 + hb + lane);
            for (int q = 0; q < CL; ++q)
              if (q != (int)rank) sas::st_cluster_f32(sas::mapa_shared(la, q), l_self);
          }
          // O^T of the unit, then this CTA's partials of the other CTAs' columns
          if (!sas::mbar_wait(&bars[B_OFULL], ounits & 1, ctl, p.status, 16)) break;
          ++ounits;
          sas::tc_fence_after();
          float* ws = p.red_ws + (size_t)cl * CL * CL * 2 * 128 * 32;
          const uint32_t rba = sas::smem_u32(&bars[rb + upar]);
          for (int j = 0; j < CL; ++j) {
            if (j == (int)rank) continue;
            uint32_t o[32];
            if (has_o) {
              sas::tmem_ld32(lane_addr + TM_O + 64 * j + hb, o);
              sas::tmem_wait_ld();
            } else {
#pragma unroll
              for (int h = 0; h < 32; ++h) o[h] = 0u;
            }
            float4* dst = reinterpret_cast<float4*>(ws + ((((size_t)j * CL + rank) * 2 + half) * 128 + gst) * 32);
#pragma unroll
            for (int h = 0; h < 32; h += 4)
              dst[h / 4] = make_float4(__uint_as_float(o[h]), __uint_as_float(o[h + 1]), __uint_as_float(o[h + 2]),
                                       __uint_as_float(o[h + 3]));
            sas::mbar_arrive_cluster(sas::mapa_shared(rba, j));
          }
          // this CTA's own columns: the partials of the other three, in rank order
          uint32_t own[32];
          if (has_o) {
            sas::tmem_ld32(lane_addr + TM_O + 64 * rank + hb, own);
            sas::tmem_wait_ld();
          } else {
#pragma unroll
            for (int h = 0; h < 32; ++h) own[h] = 0u;
          }
          sas::tc_fence_before();
          sas::mbar_arrive(&bars[B_OEMPTY]);  // O^T has been read
          if (!sas::mbar_wait_cluster(&bars[rb + upar], (runits >> 1) & 1, ctl, p.status, 17)) break;
          ++runits;
          float acc[32];
#pragma unroll
          for (int h = 0; h < 32; ++h) acc[h] = 0.f;
          for (int src = 0; src < CL; ++src) {
            if (src == (int)rank) {
#pragma unroll
              for (int h = 0; h < 32; ++h) acc[h] += __uint_as_float(own[h]);
            } else {
              const float4* sp =
                  reinterpret_cast<const float4*>(ws + ((((size_t)rank * CL + src) * 2 + half) * 128 + gst) * 32);
#pragma unroll
              for (int h = 0; h < 32; h += 4) {
                const float4 v = __ldcg(sp + h / 4);
                acc[h] += v.x;
                acc[h + 1] += v.y;
                acc[h + 2] += v.z;
                acc[h + 3] += v.w;
              }
            }
          }
          // L = sum of the CTAs' l + 2^(sink - m), lse = m + log2 L (golden.py:201-205)
          // L = sum of the CTAs' l + 2^(sink - m) for head hb + lane, summed in
          // the same order on every CTA so that all four use the same L
          float L = 0.f;
#pragma unroll
          for (int src = 0; src < CL; ++src) L += src == (int)rank ? l_self : lbuf[(upar * CL + src) * 64 + hb + lane];
          const int hl = g * HG + hb + lane;
          L += sas::ex2((hl < p.H ? p.sinks[hl] * kLog2e : 0.f) - mw[lane]);
          const float inv_l = covered ? 1.f / L : 0.f;
          if (rank == 0 && lead && hl < p.H) p.lse[(size_t)t * p.H + hl] = covered ? (mw[lane] + __log2f(L)) * kLn2 : 0.f;
          // lanes pair up (d, d^1): the even lane stores head h for both columns,
          // the odd lane head h+16 (4-byte stores)
          const bool odd = lane & 1;
          const int d_even = d0 + (gst & ~1);
#pragma unroll
          for (int h = 0; h < 16; ++h) {
            const float v0 = acc[h] * __shfl_sync(0xffffffffu, inv_l, h);
            const float v1 = acc[h + 16] * __shfl_sync(0xffffffffu, inv_l, h + 16);
            const float recv = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 1);
            const uint32_t w = odd ? Io<DT>::pack(recv, v1) : Io<DT>::pack(v0, recv);
            const int hh = odd ? h + 16 : h;
            if (g * HG + hb + hh < p.H) *reinterpret_cast<uint32_t*>(outp + (size_t)(hb + hh) * D + d_even) = w;
          }
        }
        has_o = false;
      }
      ++n;
    }
  }

  sas::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    sas::tc_fence_after();
    sas::tmem_dealloc(tmem, 512);
  }
  sas::cluster_sync();  // no CTA leaves while another may still write into it
}

int g_max_clusters[64] = {};
std::mutex g_dec_mu;

}  // namespace

namespace sas {

size_t dec_workspace_bytes(int num_sms) {
  const size_t ncl = (size_t)std::max(1, num_sms / CL);
  return ncl * CL * CL * 2 * 128 * 32 * sizeof(float);
}

// Launches the cluster decode kernel; returns SAS_OK or an SAS_ERR_* code.
int launch_cluster_decode(const CUtensorMap& tm_q, int dtype, int T, int H, int B, int S, int layout, int scenario,
                          int K, int ratio, int win_left, int ori_bs, int ori_bt_stride, int cmp_bs,
                          int cmp_bt_stride, int ori_nblk, int cmp_nblk, const void* ori_kv, const void* cmp_kv,
                          const int32_t* ori_bt, const int32_t* cmp_bt, const int32_t* idx, const int32_t* cu,
                          const int32_t* seqused_kv, const int32_t* meta, const float* sinks, float scale_log2,
                          void* out, float* lse, void* ws, int num_sms, int32_t* status, int q_box_h, bool early,
                          unsigned long long wait_ns, cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SAS_ERR_CUDA;
  DecParams p{};
  p.T = T;
  p.H = H;
  p.G = (H + HG - 1) / HG;
  p.B = B;
  p.S = S;
  p.layout = layout;
  p.scenario = scenario;
  p.K = K;
  p.ratio = ratio;
  p.win_left = win_left;
  p.ori_bs = ori_bs;
  p.ori_bt_stride = ori_bt_stride;
  p.cmp_bs = cmp_bs;
  p.cmp_bt_stride = cmp_bt_stride;
  p.ori_nblk = ori_nblk;
  p.cmp_nblk = cmp_nblk;
  p.ori_kv = static_cast<const uint8_t*>(ori_kv);
  p.cmp_kv = static_cast<const uint8_t*>(cmp_kv);
  p.ori_bt = ori_bt;
  p.cmp_bt = cmp_bt;
  p.idx = idx;
  p.cu = cu;
  p.seqused_kv = seqused_kv;
  p.meta = meta;
  p.sinks = sinks;
  p.scale_log2 = scale_log2;
  p.out = out;
  p.lse = lse;
  p.red_ws = static_cast<float*>(ws);
  p.status = status;
  p.q_box_h = q_box_h;
  p.early = early ? 1 : 0;
  p.wait_ns = wait_ns;
  auto kernel = dtype == SAS_DTYPE_BF16 ? sas_dec_kernel<0> : sas_dec_kernel<1>;
  int ncl;
  {
    std::lock_guard<std::mutex> lk(g_dec_mu);
    if (g_max_clusters[dev] == 0) {
      if (cudaFuncSetAttribute(sas_dec_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
              cudaSuccess ||
          cudaFuncSetAttribute(sas_dec_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
              cudaSuccess)
        return SAS_ERR_CUDA;
      cudaLaunchConfig_t q{};
      q.gridDim = dim3(CL * std::max(1, num_sms / CL));
      q.blockDim = dim3(kThreads);
      q.dynamicSmemBytes = SMEM_BYTES;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, sas_dec_kernel<0>, &q) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return SAS_ERR_CUDA;
      }
      g_max_clusters[dev] = n;
    }
    ncl = std::min(g_max_clusters[dev], std::max(1, num_sms / CL));
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(CL * ncl);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, tm_q, p) == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}

}  // namespace sas
