// Fused sparse shared-KV attention forward for B200 (sm_100a).
//
// Three kernels, all launched by sas_sparse_attn_sharedkv_fwd on the caller's
// stream:
//
// 1. sas_plan_kernel (1 CTA): walks the metadata's per-core windows of
//    linearised (b, s) ids exactly like the reference kernel's outer loop
//    (kernel.py:254-278: pid in [bn2_start*max_seq+m_start,
//    bn2_end*max_seq+m_end), s < act_q), and gives every covered query token
//    its work in 128-row chunks: ceil((win_left+1)/128) window chunks plus
//    ceil(n_cmp/128) compressed chunks, n_cmp = min(K, threshold) for SCFA,
//    threshold for CFA (threshold = (s_g+1)//ratio, golden.py:41-51).
//    An exclusive scan gives each token's first chunk-unit.
//
// 2. sas_fwd_kernel (persistent, R x G CTAs, one per SM): the unit sequence
//    is cut into R equal contiguous ranges; the G CTAs of a range each own
//    64 query heads (head group g) and walk the same rows, so the second
//    reader of every KV row hits L2. Per CTA, warp-specialised:
//      warp 0   producer: resolves window positions / top-k ids through the
//               block tables (kernel.py:285-401, 686-766), publishes a
//               128-bit row-validity mask and gathers the 128 rows x 512
//               cols chunk with TMA tile::gather4 in eight 64-col slabs
//               (128B swizzle); masked rows use an out-of-range row, so TMA
//               zero-fills them without touching HBM.
//      warp 1   MMA issuer (one thread): transposed attention so the KV rows
//               fill the M=128 datapath and the 64 heads are N:
//                 S^T[128 x 64]  = K[128 x 512] . Q^T          (K-major A and B)
//                 O^T[512 x 64] += V^T[512 x 128] . P^T[128 x 64] (4 MMAs of
//               M=128; V^T is the SAME smem tile read MN-major, since K=V)
//               TMEM: S^T in cols [0,64), O^T tiles in cols [64,320).
//      warps 2-5 softmax / epilogue: one thread per KV row (TMEM lane). The
//               row mask (window idx <= s_g; compressed 0 <= idx < threshold,
//               scan stopped at the first -1) sets scores to -inf; the
//               per-head running max is a warp reduce-scatter plus a 4-way
//               smem merge; the state starts at (m, l) = (sink, 1) in log2
//               units (kernel.py:594-618, golden.py:156-160) and O^T is only
//               rescaled when a head's max grows by more than 2^8. P is
//               rounded to the I/O dtype before P.V while l sums the
//               unrounded p (golden.py:191-195). Epilogue: O/l, lse = m+ln l.
//    A token whose chunks all fall in one range is finished in place
//    (sink folded in); a token cut by a range boundary leaves normalised
//    partials (o, lse2) in the workspace.
//
// 3. sas_combine_kernel: for every cut token, lse = log2(sum 2^lse_i +
//    2^sink), out = sum 2^(lse_i - lse) o_i; also zero-fills output rows of
//    tokens that have no work (BSND padding), as golden.py leaves them zero.
#include <cuda.h>
#include <cstdio>
#include <mutex>

#include "sas_common.cuh"

namespace {

constexpr int D = 512;
constexpr int HG = 64;        // heads per CTA (MMA N)
constexpr int CH = 128;       // KV rows per chunk (MMA M)
constexpr int NSLAB = 8;      // 64-column slabs per chunk
constexpr int SLAB_BYTES = CH * 128;  // 16 KB
constexpr int Q_SLAB_BYTES = HG * 128;  // 8 KB
constexpr int kLoaderWarps = 4;         // warps 0-3: cp.async loaders
constexpr int kLoaderThreads = 32 * kLoaderWarps;
constexpr int kSoftmaxWarp0 = 4;        // warps 4-7: softmax / epilogue
constexpr int kMmaWarp = 8;             // warp 8: TMEM owner and MMA issuer
constexpr int kThreads = 32 * 9;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// shared memory map (offsets from a 1024-aligned base)
constexpr int OFF_Q = 0;
constexpr int OFF_KV = OFF_Q + NSLAB * Q_SLAB_BYTES;     // 64 KB
constexpr int OFF_P = OFF_KV + NSLAB * SLAB_BYTES;       // +128 KB
constexpr int OFF_MISC = OFF_P + CH * 128;               // +16 KB
// misc region
constexpr int M_BAR = 0;         // 32 mbarriers x 8 B
constexpr int M_TMEM = 256;      // tmem base address
constexpr int M_ABORT = 260;
constexpr int M_MASK = 272;      // 2 x 4 words
constexpr int M_FIRST = 320;     // 2 x 4 ints
constexpr int M_RED = 512;       // 4 x 64 floats = 1 KB
constexpr int M_MRUN = 1536;     // 64 floats
constexpr int M_ALPHA = 1792;    // 64 floats
constexpr int M_INV = 2048;      // 64 floats
constexpr int MISC_BYTES = 2304;
constexpr int SMEM_BYTES = OFF_MISC + MISC_BYTES + 1024;  // + alignment slack

// barrier indices
constexpr int B_FULL = 0;        // 8
constexpr int B_EMPTY = 8;       // 8
constexpr int B_QFULL = 16;
constexpr int B_QEMPTY = 17;
constexpr int B_SFULL = 18;
constexpr int B_PREADY = 19;
constexpr int B_OFULL = 20;
constexpr int B_OEMPTY = 21;
constexpr int B_MFULL = 22;      // 2
constexpr int B_MEMPTY = 24;     // 2

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TM_S = 0;
constexpr uint32_t TM_O = 64;

struct TokInfo {
  int b, s_g, n_cmp, thr;
};

struct PlanParams {
  int T, B, S, layout, scenario, K, ratio, win_left, n_win_chunks;
  const int32_t* cu;
  const int32_t* seqused_kv;
  const int32_t* meta;
  TokInfo* tok;
  int32_t* unit_start;  // [T+1]
  int H, dtype_bytes;
  void* out;            // rows of tokens without work are zeroed here
  float* lse;
};

struct FwdParams {
  int T, H, G, R, scenario, K, ratio, win_left, n_win_chunks;
  int ori_bs, ori_bt_stride, cmp_bs, cmp_bt_stride;
  int ori_rows, cmp_rows;  // OOB row coordinate = row count
  const uint8_t* ori_kv;   // paged pools, rows of D elements
  const uint8_t* cmp_kv;
  const int32_t* ori_bt;
  const int32_t* cmp_bt;
  const int32_t* idx;
  const float* sinks;
  float scale_log2;
  void* out;
  float* lse;
  const TokInfo* tok;
  const int32_t* unit_start;
  float* part_o;    // [R*2*G][64][512]
  float* part_lse;  // [R*2*G][64]
  int32_t* status;
  int q_box_h;
  float tau;                 // lazy-rescale threshold, log2 units (0 = exact running max)
  unsigned long long* trace; // optional per-CTA cycle counters (nullptr in production)
};

// trace slots per CTA (SM cycles, accumulated by one thread of each role)
enum TraceSlot {
  TR_TOTAL = 0, TR_P_COORD, TR_P_WAIT_EMPTY, TR_P_WAIT_MASK, TR_P_ISSUE, TR_M_WAIT_Q, TR_M_WAIT_FULL,
  TR_M_WAIT_P, TR_M_WAIT_O, TR_S_WAIT_MASK, TR_S_WAIT_S, TR_S_SOFTMAX, TR_S_WAIT_O, TR_S_EPI, TR_CHUNKS,
  TR_SEGS, TR_E_TMEM, TR_E_STAGE, TR_E_COPY, TR_E_RED, TR_NSLOTS = 20
};

__device__ __forceinline__ int py_floordiv(int a, int b) {
  int q = a / b, r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) --q;
  return q;
}

// ------------------------------------------------------------------ plan
__global__ void __launch_bounds__(1024, 1) sas_plan_kernel(PlanParams p) {
  __shared__ int s_smax;
  __shared__ int s_lin[SAS_AIC_CORE_NUM][2];
  __shared__ int s_en[SAS_AIC_CORE_NUM];
  __shared__ int s_warp[32];
  __shared__ int s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // max_seq: the reference api's S_max (api.py:208-215 / 229)
  int mx = 0;
  if (p.layout == SAS_LAYOUT_TND) {
    for (int b = tid; b < p.B; b += blockDim.x) mx = max(mx, p.cu[b + 1] - p.cu[b]);
  } else {
    mx = p.S;
  }
  for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_warp[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    int m = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = max(m, s_warp[w]);
    s_smax = m;
    s_carry = 0;
  }
  __syncthreads();
  const int smax = s_smax;
  if (tid < SAS_AIC_CORE_NUM) {
    const int32_t* row = p.meta + tid * 8;
    s_en[tid] = row[0];
    // pid = bn2 * max_seq + m  (N2 == 1, so bn2 == b)
    s_lin[tid][0] = row[1] * smax + row[2];
    s_lin[tid][1] = row[4] * smax + row[5];
  }
  __syncthreads();
  for (int t0 = 0; t0 < p.T; t0 += blockDim.x) {
    const int t = t0 + tid;
    int units = 0;
    if (t < p.T) {
      int b, s, act_q;
      if (p.layout == SAS_LAYOUT_TND) {
        int lo = 0, hi = p.B - 1;  // last b with cu[b] <= t
        while (lo < hi) {
          int mid = (lo + hi + 1) >> 1;
          if (p.cu[mid] <= t) lo = mid; else hi = mid - 1;
        }
        b = lo;
        s = t - p.cu[b];
        act_q = p.cu[b + 1] - p.cu[b];
      } else {
        b = t / p.S;
        s = t - b * p.S;
        act_q = p.cu ? p.cu[b + 1] - p.cu[b] : p.S;
      }
      TokInfo ti{b, 0, 0, 0};
      if (s < act_q && b < p.B) {
        const int pid = b * smax + s;
        bool covered = false;
        for (int i = 0; i < SAS_AIC_CORE_NUM; ++i)
          covered |= (s_en[i] != 0) && pid >= s_lin[i][0] && pid < s_lin[i][1];
        const int act_kv = p.seqused_kv[b];
        const int s_g = act_kv - act_q + s;
        const int thr = max(py_floordiv(s_g + 1, p.ratio), 0);
        int n_cmp = 0;
        if (p.scenario == 3) n_cmp = min(p.K, thr);
        else if (p.scenario == 2) n_cmp = thr;
        ti.s_g = s_g;
        ti.n_cmp = n_cmp;
        ti.thr = thr;
        if (covered) units = p.n_win_chunks + (n_cmp + CH - 1) / CH;
      }
      p.tok[t] = ti;
      if (units == 0) {
        // padding / uncovered token: zero output and LSE (golden.py leaves them zero)
        uint4* o = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + (size_t)t * p.H * D * p.dtype_bytes);
        for (int i = 0; i < p.H * D * p.dtype_bytes / 16; ++i) o[i] = make_uint4(0, 0, 0, 0);
        if (p.lse)
          for (int h = 0; h < p.H; ++h) p.lse[(size_t)t * p.H + h] = 0.f;
      }
    }
    // block exclusive scan of units
    int v = units;
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (lane == 31) s_warp[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int w = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : 0;
      for (int o = 1; o < 32; o <<= 1) {
        int u = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += u;
      }
      s_warp[lane] = w;
    }
    __syncthreads();
    const int excl = s_carry + (warp ? s_warp[warp - 1] : 0) + v - units;
    if (t < p.T) p.unit_start[t] = excl;
    __syncthreads();
    if (tid == 0) s_carry += s_warp[31];
    __syncthreads();
  }
  if (tid == 0) p.unit_start[p.T] = s_carry;
}

// ------------------------------------------------------- work enumeration
struct Seg {
  int t, cb, ce, units, which;
  bool complete;
};

struct Walker {
  int pos, end, t, u0;
  const int32_t* us;
  __device__ void init(const int32_t* unit_start, int T, int R, int r) {
    us = unit_start;
    const int U = us[T];
    const int u = (U + R - 1) / R;
    u0 = min(r * u, U);
    pos = u0;
    end = min(u0 + u, U);
    // largest t with unit_start[t] <= u0
    int lo = 0, hi = T - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (us[mid] <= u0) lo = mid; else hi = mid - 1;
    }
    t = lo;
  }
  __device__ bool next(Seg& s) {
    if (pos >= end) return false;
    while (us[t + 1] <= pos) ++t;  // skip tokens without units
    const int st = us[t], n = us[t + 1] - st;
    s.t = t;
    s.units = n;
    s.cb = pos - st;
    s.ce = min(st + n, end) - st;
    s.complete = (s.cb == 0 && s.ce == n);
    s.which = (pos == u0) ? 0 : 1;
    pos = st + s.ce;
    ++t;
    return true;
  }
};

template <int DT>
struct IoType;
template <>
struct IoType<0> {
  using T = __nv_bfloat16;
  __device__ static uint32_t pack(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ static uint16_t one(float a) {
    __nv_bfloat16 v = __float2bfloat16_rn(a);
    return *reinterpret_cast<uint16_t*>(&v);
  }
};
template <>
struct IoType<1> {
  using T = __half;
  __device__ static uint32_t pack(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ static uint16_t one(float a) {
    __half v = __float2half_rn(a);
    return *reinterpret_cast<uint16_t*>(&v);
  }
};

// Reduce 64 per-thread values across the 32 lanes of a warp; afterwards
// v[0], v[1] hold the reduction for columns 2*lane and 2*lane+1.
template <bool IS_MAX>
__device__ __forceinline__ void warp_reduce_scatter64(float (&v)[64], int lane) {
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    const int half = 32 >> step;
    const int m = 16 >> step;
    const bool up = (lane & m) != 0;
#pragma unroll
    for (int k = 0; k < half; ++k) {
      const float a = v[k], b = v[k + half];
      const float send = up ? a : b;
      const float keep = up ? b : a;
      const float recv = __shfl_xor_sync(0xffffffffu, send, m);
      v[k] = IS_MAX ? fmaxf(keep, recv) : keep + recv;
    }
  }
}

__device__ __forceinline__ bool twait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                      int where, bool tracing, unsigned long long& acc) {
  const long long t0 = tracing ? clock64() : 0;
  const bool r = sas::mbar_wait(bar, parity, abort_flag, status, where);
  if (tracing) acc += clock64() - t0;
  return r;
}

// 16-byte async copy global -> shared; src_bytes = 0 writes zeros without reading.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// Arrive on `bar` once every cp.async issued so far by this thread has landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(sas::smem_u32(bar)) : "memory");
}

template <int DT>
__global__ void __launch_bounds__(kThreads, 1)
    sas_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const FwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = sas::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  uint8_t* misc = smem + OFF_MISC;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + M_BAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + M_ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + M_TMEM);
  uint32_t* mask_words = reinterpret_cast<uint32_t*>(misc + M_MASK);    // [2][4]
  int* first_neg = reinterpret_cast<int*>(misc + M_FIRST);               // [2][4]
  float* red = reinterpret_cast<float*>(misc + M_RED);
  float* m_run = reinterpret_cast<float*>(misc + M_MRUN);
  float* alpha_s = reinterpret_cast<float*>(misc + M_ALPHA);
  float* inv_s = reinterpret_cast<float*>(misc + M_INV);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = blockIdx.x / p.G, g = blockIdx.x % p.G;

  if (tid == 0) {
    for (int i = 0; i < NSLAB; ++i) {
      sas::mbar_init(&bars[B_FULL + i], kLoaderThreads);
      sas::mbar_init(&bars[B_EMPTY + i], 1);
    }
    sas::mbar_init(&bars[B_QFULL], 1);
    sas::mbar_init(&bars[B_QEMPTY], 1);
    sas::mbar_init(&bars[B_SFULL], 1);
    sas::mbar_init(&bars[B_PREADY], 128);
    sas::mbar_init(&bars[B_OFULL], 1);
    sas::mbar_init(&bars[B_OEMPTY], 128);
    for (int i = 0; i < 2; ++i) {
      sas::mbar_init(&bars[B_MFULL + i], kLoaderThreads / 32);
      sas::mbar_init(&bars[B_MEMPTY + i], 128);
    }
    *abort_flag = 0;
    sas::fence_mbar_init();
  }
  // heads beyond the Q box stay zero in every slab (H < 64)
  if (p.q_box_h < HG) {
    for (int i = tid; i < NSLAB * Q_SLAB_BYTES / 16; i += kThreads)
      reinterpret_cast<uint4*>(smem + OFF_Q)[i] = make_uint4(0, 0, 0, 0);
    sas::fence_proxy_async_smem();
  }
  if (warp == kMmaWarp) {
    sas::tmem_alloc(tmem_slot, TMEM_COLS);
    sas::tmem_relinquish();
  }
  if (tid == 0) sas::tma_prefetch_desc(&tm_q);
  sas::tc_fence_before();
  __syncthreads();
  sas::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool tracing = p.trace != nullptr;
  unsigned long long tr[TR_NSLOTS];
#pragma unroll
  for (int i = 0; i < TR_NSLOTS; ++i) tr[i] = 0;
  const long long t_start = tracing ? clock64() : 0;

  if (warp < kLoaderWarps) {
    // =============================== loaders: one KV row per thread per chunk
    const int lw = warp;                // rows [32*lw, 32*lw+32) of every chunk
    const int row = lw * 32 + lane;
    const int sub = lane >> 3, c16 = lane & 7;
    const uint32_t kv_base = sas::smem_u32(smem + OFF_KV);
    Walker wk;
    wk.init(p.unit_start, p.T, p.R, r);
    Seg sg;
    uint32_t gchunk = 0, seg_i = 0;
    const uint32_t q_bytes = (uint32_t)NSLAB * p.q_box_h * 128;
    bool ok = true;
    while (ok && wk.next(sg)) {
      const TokInfo ti = p.tok[sg.t];
      if (tid == 0) {
        if (!twait(&bars[B_QEMPTY], (seg_i & 1) ^ 1, abort_flag, p.status, 1, tracing, tr[TR_P_WAIT_EMPTY])) {
          ok = false;
        } else {
          sas::mbar_arrive_expect_tx(&bars[B_QFULL], q_bytes);
          for (int s = 0; s < NSLAB; ++s)
            sas::tma_load_3d(smem + OFF_Q + s * Q_SLAB_BYTES, &tm_q, &bars[B_QFULL], s * 64, g * HG, sg.t);
        }
      }
      // the compressed scan stops at the first -1 (golden.py:55-56): a range
      // that starts inside a token looks for one in the slots before it
      bool stopped = false;
      const int cmp_c0 = max(sg.cb - p.n_win_chunks, 0);
      if (p.scenario == 3 && cmp_c0 > 0) {
        const int lim = min(cmp_c0 * CH, ti.n_cmp);
        const int32_t* ip = p.idx + (size_t)sg.t * p.K;
        int neg = 0;
        for (int e = row; e < lim; e += kLoaderThreads) neg |= (ip[e] == -1);
        stopped = sas::named_bar_or(3, kLoaderThreads, neg) != 0;
      }
      for (int c = sg.cb; ok && c < sg.ce; ++c, ++gchunk) {
        const long long tc0 = tracing ? clock64() : 0;
        const bool is_win = c < p.n_win_chunks;
        long long coord = -1;  // physical row in the pool, -1 = masked
        bool val;
        if (is_win) {
          const int lo = max(ti.s_g - p.win_left, 0);
          const int pos = lo + c * CH + row;
          val = (ti.s_g >= 0) && pos <= ti.s_g;
          if (val) {
            const int blk = p.ori_bt[(size_t)ti.b * p.ori_bt_stride + pos / p.ori_bs];
            val = blk >= 0;
            coord = (long long)blk * p.ori_bs + pos % p.ori_bs;
          }
        } else {
          const int e = (c - p.n_win_chunks) * CH + row;
          val = e < ti.n_cmp;
          int id = e;
          if (p.scenario == 3) {
            id = val ? p.idx[(size_t)sg.t * p.K + e] : 0;
            const unsigned bal = __ballot_sync(0xffffffffu, val && id == -1);
            if (lane == 0) first_neg[(gchunk & 1) * 4 + lw] = bal ? lw * 32 + __ffs(bal) - 1 : CH;
            sas::named_bar_sync(3, kLoaderThreads);
            const int* fn = first_neg + (gchunk & 1) * 4;
            const int cf = min(min(fn[0], fn[1]), min(fn[2], fn[3]));
            val = val && !stopped && row < cf && id >= 0 && id < ti.thr;
            stopped = stopped || cf < CH;
          } else {
            val = val && id < ti.thr;
          }
          if (val) {
            const int blk = p.cmp_bt[(size_t)ti.b * p.cmp_bt_stride + id / p.cmp_bs];
            val = blk >= 0;
            coord = (long long)blk * p.cmp_bs + id % p.cmp_bs;
          }
        }
        if (!val) coord = -1;
        if (tracing) tr[TR_P_COORD] += clock64() - tc0;
        // ---- publish the validity mask of this chunk
        const int mb = gchunk & 1;
        if (!twait(&bars[B_MEMPTY + mb], ((gchunk >> 1) & 1) ^ 1, abort_flag, p.status, 2, tracing,
                   tr[TR_P_WAIT_MASK])) {
          ok = false;
          break;
        }
        const unsigned vb = __ballot_sync(0xffffffffu, val);
        if (lane == 0) {
          mask_words[mb * 4 + lw] = vb;
          sas::mbar_arrive(&bars[B_MFULL + mb]);
        }
        // ---- rows this lane copies: 4 rows x 8 lanes x 16 B per instruction
        long long crw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) crw[i] = __shfl_sync(0xffffffffu, coord, 4 * i + sub);
        const uint8_t* pool = is_win ? p.ori_kv : p.cmp_kv;
        for (int s = 0; s < NSLAB; ++s) {
          if (!twait(&bars[B_EMPTY + s], (gchunk & 1) ^ 1, abort_flag, p.status, 3, tracing,
                     tr[TR_P_WAIT_EMPTY])) {
            ok = false;
            break;
          }
          const uint32_t slab = kv_base + s * SLAB_BYTES;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rl = 4 * i + sub;
            const uint32_t dst = slab + (lw * 32 + rl) * 128 + ((c16 ^ (rl & 7)) << 4);
            const bool v = crw[i] >= 0;
            const uint8_t* src = pool + (size_t)(v ? crw[i] : 0) * (D * 2) + s * 128 + c16 * 16;
            cp_async16(dst, src, v ? 16u : 0u);
          }
          cp_async_arrive(&bars[B_FULL + s]);
        }
      }
      ++seg_i;
    }
  } else if (warp == kMmaWarp) {
    // =============================== MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc1 = sas::umma_idesc_f16(DT == 0 ? 1 : 0, 128, HG, 0, 0);
      constexpr uint32_t idesc2 = sas::umma_idesc_f16(DT == 0 ? 1 : 0, 128, HG, 1, 1);
      const uint32_t q_base = sas::smem_u32(smem + OFF_Q);
      const uint32_t kv_base = sas::smem_u32(smem + OFF_KV);
      const uint32_t p_base = sas::smem_u32(smem + OFF_P);
      Walker wk;
      wk.init(p.unit_start, p.T, p.R, r);
      Seg sg;
      uint32_t gchunk = 0, seg_i = 0;
      bool ok = true;
      while (ok && wk.next(sg)) {
        if (!twait(&bars[B_QFULL], seg_i & 1, abort_flag, p.status, 4, tracing, tr[TR_M_WAIT_Q])) break;
        for (int c = sg.cb; c < sg.ce; ++c, ++gchunk) {
          const bool first = c == sg.cb, last = c == sg.ce - 1;
          // S^T = K . Q^T
          for (int s = 0; s < NSLAB; ++s) {
            if (!twait(&bars[B_FULL + s], gchunk & 1, abort_flag, p.status, 5, tracing, tr[TR_M_WAIT_FULL])) {
              ok = false;
              break;
            }
            sas::fence_proxy_async_smem();  // cp.async (generic proxy) writes -> tensor-core reads
            sas::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sas::umma_desc_sw128(kv_base + s * SLAB_BYTES + kk * 32, 16, 1024);
              const uint64_t bd = sas::umma_desc_sw128(q_base + s * Q_SLAB_BYTES + kk * 32, 16, 1024);
              sas::umma_ss(tmem + TM_S, ad, bd, idesc1, (s | kk) != 0);
            }
          }
          if (!ok) break;
          sas::umma_commit(&bars[B_SFULL]);
          if (last) sas::umma_commit(&bars[B_QEMPTY]);
          // O^T += V^T . P^T
          if (!twait(&bars[B_PREADY], gchunk & 1, abort_flag, p.status, 6, tracing, tr[TR_M_WAIT_P])) {
            ok = false;
            break;
          }
          if (first && seg_i > 0) {
            if (!twait(&bars[B_OEMPTY], (seg_i - 1) & 1, abort_flag, p.status, 7, tracing, tr[TR_M_WAIT_O])) {
              ok = false;
              break;
            }
          }
          sas::tc_fence_after();
#pragma unroll 1
          for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t ad = sas::umma_desc_sw128(kv_base + (2 * j) * SLAB_BYTES + kk * 2048, SLAB_BYTES, 1024);
              const uint64_t bd = sas::umma_desc_sw128(p_base + kk * 2048, 8192, 1024);
              sas::umma_ss(tmem + TM_O + 64 * j, ad, bd, idesc2, (first && kk == 0) ? 0u : 1u);
            }
            sas::umma_commit(&bars[B_EMPTY + 2 * j]);
            sas::umma_commit(&bars[B_EMPTY + 2 * j + 1]);
          }
          if (last) sas::umma_commit(&bars[B_OFULL]);
        }
        ++seg_i;
      }
    }
    __syncwarp();
  } else if (warp >= kSoftmaxWarp0 && warp < kSoftmaxWarp0 + 4) {
    // =============================== softmax / epilogue (one thread per KV row)
    using IO = IoType<DT>;
    const int quad = warp & 3;          // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;   // KV row of the chunk / d within an O^T tile
    const int st = tid - kSoftmaxWarp0 * 32;  // 0..127
    const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
    float lsum0 = 0.f, lsum1 = 0.f;  // running sums of heads 2*lane, 2*lane+1 over this warp's rows
    Walker wk;
    wk.init(p.unit_start, p.T, p.R, r);
    Seg sg;
    uint32_t gchunk = 0, seg_i = 0;
    bool ok = true;
    uint8_t* pbuf = smem + OFF_P;
    while (ok && wk.next(sg)) {
      const int h0 = g * HG;
      if (st < HG) {
        const int h = h0 + st;
        m_run[st] = h < p.H ? p.sinks[h] * kLog2e : 0.f;
      }
      lsum0 = lsum1 = 0.f;
      for (int c = sg.cb; c < sg.ce; ++c, ++gchunk) {
        const bool first = c == sg.cb, last = c == sg.ce - 1;
        const int mb = gchunk & 1;
        if (!twait(&bars[B_MFULL + mb], (gchunk >> 1) & 1, abort_flag, p.status, 8, tracing, tr[TR_S_WAIT_MASK])) {
          ok = false;
          break;
        }
        const bool valid = (mask_words[mb * 4 + (row >> 5)] >> (row & 31)) & 1;
        sas::mbar_arrive(&bars[B_MEMPTY + mb]);
        if (!twait(&bars[B_SFULL], gchunk & 1, abort_flag, p.status, 9, tracing, tr[TR_S_WAIT_S])) {
          ok = false;
          break;
        }
        sas::tc_fence_after();
        const long long ts0 = tracing ? clock64() : 0;
        // ---- this row's scaled scores (log2 units), one TMEM read per chunk
        float x[64];
        {
          uint32_t ra[32], rb[32];
          sas::tmem_ld32(lane_addr + TM_S, ra);
          sas::tmem_ld32(lane_addr + TM_S + 32, rb);
          sas::tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < 32; ++h) {
            x[h] = valid ? __uint_as_float(ra[h]) * p.scale_log2 : -INFINITY;
            x[h + 32] = valid ? __uint_as_float(rb[h]) * p.scale_log2 : -INFINITY;
          }
        }
        // ---- per-head max over the warp's 32 rows (redux), then over the 4 warps
#pragma unroll
        for (int h = 0; h < 64; h += 4) {
          float4 w;
          w.x = sas::warp_max_f32(x[h]);
          w.y = sas::warp_max_f32(x[h + 1]);
          w.z = sas::warp_max_f32(x[h + 2]);
          w.w = sas::warp_max_f32(x[h + 3]);
          if (lane == 0) *reinterpret_cast<float4*>(red + quad * 64 + h) = w;
        }
        sas::named_bar_sync(1, 128);
        int need = 0;
        if (st < HG) {
          const float mx = fmaxf(fmaxf(red[st], red[64 + st]), fmaxf(red[128 + st], red[192 + st]));
          const float mo = m_run[st];
          float al = 1.f;
          if (mx > mo + p.tau) {
            al = sas::ex2(mo - mx);
            m_run[st] = mx;
            need = 1;
          }
          alpha_s[st] = al;
        }
        need = sas::named_bar_or(2, 128, need);
        if (need) {
          lsum0 *= alpha_s[2 * lane];
          lsum1 *= alpha_s[2 * lane + 1];
          if (!first) {
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
              uint32_t o[32];
              sas::tmem_ld32(lane_addr + TM_O + 32 * j, o);
              sas::tmem_wait_ld();
              const int hb = (j & 1) * 32;
#pragma unroll
              for (int h = 0; h < 32; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha_s[hb + h]);
              sas::tmem_st32(lane_addr + TM_O + 32 * j, o);
            }
            sas::tmem_wait_st();
          }
        }
        // ---- p = 2^(x - m) (masked rows give 0); P^T to smem (128 B rows,
        // 128B swizzle) rounded to the I/O dtype; l sums the unrounded p
        {
#pragma unroll
          for (int h = 0; h < 64; ++h) x[h] = sas::ex2(x[h] - m_run[h]);
          uint8_t* prow = pbuf + row * 128;
#pragma unroll
          for (int c16 = 0; c16 < 8; ++c16) {
            const int h = c16 * 8;
            *reinterpret_cast<uint4*>(prow + ((c16 ^ (row & 7)) << 4)) =
                make_uint4(IO::pack(x[h], x[h + 1]), IO::pack(x[h + 2], x[h + 3]),
                           IO::pack(x[h + 4], x[h + 5]), IO::pack(x[h + 6], x[h + 7]));
          }
          warp_reduce_scatter64<false>(x, lane);
          lsum0 += x[0];
          lsum1 += x[1];
        }
        sas::fence_proxy_async_smem();
        sas::tc_fence_before();
        sas::mbar_arrive(&bars[B_PREADY]);
        if (tracing) {
          tr[TR_S_SOFTMAX] += clock64() - ts0;
          tr[TR_CHUNKS] += 1;
        }

        if (last) {
          // ------------------------------ epilogue
          if (!twait(&bars[B_OFULL], seg_i & 1, abort_flag, p.status, 10, tracing, tr[TR_S_WAIT_O])) {
            ok = false;
            break;
          }
          sas::tc_fence_after();
          const long long te0 = tracing ? clock64() : 0;
          red[quad * 64 + 2 * lane] = lsum0;
          red[quad * 64 + 2 * lane + 1] = lsum1;
          sas::named_bar_sync(1, 128);
          if (st < HG) {
            const int h = h0 + st;
            const float L = red[st] + red[64 + st] + red[128 + st] + red[192 + st];
            const float m = m_run[st];
            if (sg.complete) {
              const float sink = h < p.H ? p.sinks[h] * kLog2e : 0.f;
              const float Lf = L + sas::ex2(sink - m);
              inv_s[st] = 1.f / Lf;
              if (p.lse && h < p.H) p.lse[(size_t)sg.t * p.H + h] = (m + __log2f(Lf)) * kLn2;
            } else {
              inv_s[st] = L > 0.f ? 1.f / L : 0.f;
              const size_t slot = ((size_t)r * 2 + sg.which) * p.G + g;
              p.part_lse[slot * HG + st] = L > 0.f ? m + __log2f(L) : -INFINITY;
            }
          }
          sas::named_bar_sync(1, 128);
          if (tracing) tr[TR_E_RED] += clock64() - te0;
          if (sg.complete) {
            // direct stores: lanes pair up (row, row^1); the even lane stores
            // head h for both rows, the odd lane head h+32 (4-byte stores, two
            // 64-byte runs per warp instruction; no shared-memory staging, which
            // would compete with the next segment's MMA operand reads)
            typename IO::T* outp = reinterpret_cast<typename IO::T*>(p.out) + (size_t)sg.t * p.H * D;
            const bool odd = lane & 1;
            const int d_even = row & ~1;
            for (int j = 0; j < 4; ++j) {
              uint32_t oa[32], ob[32];
              const long long tt0 = tracing ? clock64() : 0;
              sas::tmem_ld32(lane_addr + TM_O + 64 * j, oa);
              sas::tmem_ld32(lane_addr + TM_O + 64 * j + 32, ob);
              sas::tmem_wait_ld();
              const long long tt1 = tracing ? clock64() : 0;
              if (tracing) tr[TR_E_TMEM] += tt1 - tt0;
#pragma unroll
              for (int h = 0; h < 32; ++h) {
                const float v0 = __uint_as_float(oa[h]) * inv_s[h];
                const float v1 = __uint_as_float(ob[h]) * inv_s[h + 32];
                const float recv = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 1);
                const uint32_t w = odd ? IO::pack(recv, v1) : IO::pack(v0, recv);
                const int hh = h0 + (odd ? h + 32 : h);
                if (hh < p.H)
                  *reinterpret_cast<uint32_t*>(outp + (size_t)hh * D + j * 128 + d_even) = w;
              }
              if (tracing) tr[TR_E_STAGE] += clock64() - tt1;
            }
          } else {
            const size_t slot = ((size_t)r * 2 + sg.which) * p.G + g;
            float* po = p.part_o + slot * HG * D;
            for (int j = 0; j < 4; ++j) {
              uint32_t oa[32], ob[32];
              sas::tmem_ld32(lane_addr + TM_O + 64 * j, oa);
              sas::tmem_ld32(lane_addr + TM_O + 64 * j + 32, ob);
              sas::tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < 32; ++h) {
                po[(size_t)h * D + j * 128 + row] = __uint_as_float(oa[h]) * inv_s[h];
                po[(size_t)(h + 32) * D + j * 128 + row] = __uint_as_float(ob[h]) * inv_s[h + 32];
              }
            }
          }
          sas::tc_fence_before();
          sas::mbar_arrive(&bars[B_OEMPTY]);
          if (tracing) {
            tr[TR_S_EPI] += clock64() - te0;
            tr[TR_SEGS] += 1;
          }
        }
      }
      ++seg_i;
    }
  }

  if (tracing) {
    unsigned long long* tp = p.trace + (size_t)blockIdx.x * TR_NSLOTS;
    if (tid == 0) {
      tp[TR_P_COORD] = tr[TR_P_COORD];
      tp[TR_P_WAIT_EMPTY] = tr[TR_P_WAIT_EMPTY];
      tp[TR_P_WAIT_MASK] = tr[TR_P_WAIT_MASK];
    } else if (warp == kMmaWarp && lane == 0) {
      tp[TR_M_WAIT_Q] = tr[TR_M_WAIT_Q];
      tp[TR_M_WAIT_FULL] = tr[TR_M_WAIT_FULL];
      tp[TR_M_WAIT_P] = tr[TR_M_WAIT_P];
      tp[TR_M_WAIT_O] = tr[TR_M_WAIT_O];
    } else if (tid == kSoftmaxWarp0 * 32) {
      tp[TR_S_WAIT_MASK] = tr[TR_S_WAIT_MASK];
      tp[TR_S_WAIT_S] = tr[TR_S_WAIT_S];
      tp[TR_S_SOFTMAX] = tr[TR_S_SOFTMAX];
      tp[TR_S_WAIT_O] = tr[TR_S_WAIT_O];
      tp[TR_S_EPI] = tr[TR_S_EPI];
      tp[TR_CHUNKS] = tr[TR_CHUNKS];
      tp[TR_SEGS] = tr[TR_SEGS];
      tp[TR_TOTAL] = clock64() - t_start;
      tp[TR_E_TMEM] = tr[TR_E_TMEM];
      tp[TR_E_STAGE] = tr[TR_E_STAGE];
      tp[TR_E_COPY] = tr[TR_E_COPY];
      tp[TR_E_RED] = tr[TR_E_RED];
    }
  }
  sas::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    sas::tc_fence_after();
    sas::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// --------------------------------------------------------------- combine
// Grid (R, H): CTA (r, h) looks at the boundary of range r (unit r*u). If the
// boundary cuts a token and is the first boundary inside it, the CTA merges
// that token's partials for head h; 128 threads, 4 output columns each.
template <int DT>
__global__ void __launch_bounds__(128) sas_combine_kernel(const FwdParams p) {
  using IO = IoType<DT>;
  const int rb = blockIdx.x;
  const int h = blockIdx.y;
  if (h >= p.H || rb == 0) return;
  const int U = p.unit_start[p.T];
  const int u = (U + p.R - 1) / p.R;
  const int b0 = rb * u;
  if (b0 >= U) return;
  int lo = 0, hi = p.T - 1;  // token holding unit b0: largest t with unit_start[t] <= b0
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.unit_start[mid] <= b0) lo = mid; else hi = mid - 1;
  }
  const int t = lo;
  const int st = p.unit_start[t], n = p.unit_start[t + 1] - st;
  if (b0 == st || (rb - 1) * u > st) return;  // not a cut, or an earlier boundary owns it
  const int g = h / HG, hh = h % HG;
  typename IO::T* outp = reinterpret_cast<typename IO::T*>(p.out) + ((size_t)t * p.H + h) * D;
  const int d4 = threadIdx.x;  // float4 column group
  const int r0 = st / u, r1 = (st + n - 1) / u;
  const float sink = p.sinks[h] * kLog2e;
  constexpr int kMaxUnrolled = 8;
  float lse_i[kMaxUnrolled];
  size_t slot_i[kMaxUnrolled];
  const int ns = r1 - r0 + 1;
  float m = sink;
  for (int i = 0; i < ns; ++i) {
    const int rr = r0 + i;
    const int which = (rr == r0 && rr * u < st) ? 1 : 0;
    const size_t slot = ((size_t)rr * 2 + which) * p.G + g;
    const float l = p.part_lse[slot * HG + hh];
    if (i < kMaxUnrolled) {
      lse_i[i] = l;
      slot_i[i] = slot;
    }
    m = fmaxf(m, l);
  }
  float den = sas::ex2(sink - m);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kMaxUnrolled; ++i) {
    if (i < ns) {
      const float w = sas::ex2(lse_i[i] - m);
      den += w;
      const float4 v = reinterpret_cast<const float4*>(p.part_o + (slot_i[i] * HG + hh) * D)[d4];
      acc.x += w * v.x;
      acc.y += w * v.y;
      acc.z += w * v.z;
      acc.w += w * v.w;
    }
  }
  for (int i = kMaxUnrolled; i < ns; ++i) {  // long splits (rare): no unrolling
    const int rr = r0 + i;
    const size_t slot = ((size_t)rr * 2) * p.G + g;
    const float w = sas::ex2(p.part_lse[slot * HG + hh] - m);
    den += w;
    const float4 v = reinterpret_cast<const float4*>(p.part_o + (slot * HG + hh) * D)[d4];
    acc.x += w * v.x;
    acc.y += w * v.y;
    acc.z += w * v.z;
    acc.w += w * v.w;
  }
  const float id = 1.f / den;
  uint2 o;
  o.x = IO::pack(acc.x * id, acc.y * id);
  o.y = IO::pack(acc.z * id, acc.w * id);
  reinterpret_cast<uint2*>(outp)[d4] = o;
  if (p.lse && threadIdx.x == 0) p.lse[(size_t)t * p.H + h] = (m + __log2f(den)) * kLn2;
}

// ------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

bool make_q_map(CUtensorMap* m, const void* base, int T, int H, int box_h, CUtensorMapDataType dt) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)H * D * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_h, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Tuning / diagnostics knobs set through sas_fwd_set_option (process-wide).
float g_tau = 8.0f;
unsigned long long* g_trace = nullptr;

struct WsLayout {
  size_t tok, unit, po, pl, total;
};
WsLayout ws_layout(int T, int H, int num_sms) {
  const int G = (H + HG - 1) / HG;
  const int R = std::max(1, num_sms / G);
  WsLayout w;
  w.tok = 0;
  w.unit = align_up(w.tok + sizeof(TokInfo) * (size_t)std::max(T, 1), 256);
  w.po = align_up(w.unit + sizeof(int32_t) * ((size_t)T + 1), 256);
  w.pl = align_up(w.po + sizeof(float) * (size_t)R * 2 * G * HG * D, 256);
  w.total = align_up(w.pl + sizeof(float) * (size_t)R * 2 * G * HG, 256);
  return w;
}

}  // namespace

extern "C" int sas_version(void) { return 1; }

extern "C" int sas_fwd_set_option(int32_t option, double value, void* ptr) {
  switch (option) {
    case SAS_OPT_RESCALE_THRESHOLD:
      if (!(value >= 0.0 && value <= 64.0)) return SAS_ERR_INVALID_ARG;
      g_tau = (float)value;
      return SAS_OK;
    case SAS_OPT_TRACE_BUFFER:
      g_trace = static_cast<unsigned long long*>(ptr);
      return SAS_OK;
    default:
      return SAS_ERR_INVALID_ARG;
  }
}

extern "C" size_t sas_fwd_workspace_bytes(int32_t num_tokens, int32_t num_heads, int32_t num_sms) {
  return ws_layout(num_tokens, num_heads, num_sms).total;
}

extern "C" int sas_sparse_attn_sharedkv_fwd(
    const void* q, int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t dtype, int32_t layout_q,
    int32_t batch, int32_t max_seqlen_q, const int32_t* cu_seqlens_q, const int32_t* seqused_kv, const void* ori_kv,
    int64_t ori_num_blocks, int32_t ori_block_size, const int32_t* ori_block_table, int32_t ori_table_stride,
    const void* cmp_kv, int64_t cmp_num_blocks, int32_t cmp_block_size, const int32_t* cmp_block_table,
    int32_t cmp_table_stride, const int32_t* cmp_sparse_indices, int32_t topk, const float* sinks,
    const int32_t* metadata, float softmax_scale, int32_t cmp_ratio, int32_t ori_win_left, int32_t scenario,
    void* out, float* lse, int32_t num_sms, int32_t stage_mask, int32_t* status, void* workspace,
    size_t workspace_bytes, void* stream) {
  if (head_dim != D) return SAS_ERR_UNSUPPORTED;
  if (num_heads <= 0 || num_heads % 8 != 0) return SAS_ERR_UNSUPPORTED;
  if (dtype != SAS_DTYPE_BF16 && dtype != SAS_DTYPE_FP16) return SAS_ERR_UNSUPPORTED;
  if (scenario < 1 || scenario > 3) return SAS_ERR_INVALID_ARG;
  if (num_tokens < 0 || batch < 0 || !q || !out || !seqused_kv || !ori_kv || !ori_block_table || !sinks ||
      !metadata)
    return SAS_ERR_INVALID_ARG;
  if (layout_q == SAS_LAYOUT_TND && !cu_seqlens_q) return SAS_ERR_INVALID_ARG;
  if (layout_q == SAS_LAYOUT_BSND && (int64_t)batch * max_seqlen_q != num_tokens) return SAS_ERR_INVALID_ARG;
  if (layout_q != SAS_LAYOUT_TND && layout_q != SAS_LAYOUT_BSND) return SAS_ERR_UNSUPPORTED;
  if (ori_win_left < 0) return SAS_ERR_UNSUPPORTED;
  if (scenario >= 2 && (!cmp_kv || !cmp_block_table || cmp_ratio <= 0)) return SAS_ERR_INVALID_ARG;
  if (scenario == 3 && (!cmp_sparse_indices || topk <= 0)) return SAS_ERR_INVALID_ARG;
  if (ori_block_size <= 0 || (scenario >= 2 && cmp_block_size <= 0)) return SAS_ERR_INVALID_ARG;
  if ((int64_t)ori_num_blocks * ori_block_size >= (1LL << 31) ||
      (scenario >= 2 && (int64_t)cmp_num_blocks * cmp_block_size >= (1LL << 31)))
    return SAS_ERR_UNSUPPORTED;
  if (!sas::select_device_of(q)) return SAS_ERR_INVALID_ARG;
  if (num_sms <= 0) num_sms = 148;
  if (num_tokens == 0 || batch == 0) return SAS_OK;
  const WsLayout wl = ws_layout(num_tokens, num_heads, num_sms);
  if (!workspace || workspace_bytes < wl.total) return SAS_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);

  const int G = (num_heads + HG - 1) / HG;
  const int R = std::max(1, num_sms / G);
  const int n_win_chunks = (ori_win_left + 1 + CH - 1) / CH;

  PlanParams pp{};
  pp.T = num_tokens;
  pp.B = batch;
  pp.S = max_seqlen_q;
  pp.layout = layout_q;
  pp.scenario = scenario;
  pp.K = scenario == 3 ? topk : 0;
  pp.ratio = scenario >= 2 ? cmp_ratio : 1;
  pp.win_left = ori_win_left;
  pp.n_win_chunks = n_win_chunks;
  pp.cu = cu_seqlens_q;
  pp.seqused_kv = seqused_kv;
  pp.meta = metadata;
  pp.tok = reinterpret_cast<TokInfo*>(ws + wl.tok);
  pp.unit_start = reinterpret_cast<int32_t*>(ws + wl.unit);
  pp.H = num_heads;
  pp.dtype_bytes = 2;
  pp.out = out;
  pp.lse = lse;
  if (stage_mask & SAS_STAGE_PLAN) {
    sas_plan_kernel<<<1, 1024, 0, st>>>(pp);
    if (cudaGetLastError() != cudaSuccess) return SAS_ERR_CUDA;
  }
  if (!(stage_mask & (SAS_STAGE_ATTENTION | SAS_STAGE_COMBINE))) return SAS_OK;

  const CUtensorMapDataType tdt = dtype == SAS_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  alignas(64) CUtensorMap tm_q;
  const int q_box_h = std::min(HG, num_heads);
  const int64_t ori_rows = ori_num_blocks * ori_block_size;
  const int64_t cmp_rows = scenario >= 2 ? cmp_num_blocks * cmp_block_size : 0;
  if (!make_q_map(&tm_q, q, num_tokens, num_heads, q_box_h, tdt)) return SAS_ERR_CUDA;

  FwdParams fp{};
  fp.T = num_tokens;
  fp.H = num_heads;
  fp.G = G;
  fp.R = R;
  fp.scenario = scenario;
  fp.K = scenario == 3 ? topk : 0;
  fp.ratio = pp.ratio;
  fp.win_left = ori_win_left;
  fp.n_win_chunks = n_win_chunks;
  fp.ori_bs = ori_block_size;
  fp.ori_bt_stride = ori_table_stride;
  fp.cmp_bs = scenario >= 2 ? cmp_block_size : 1;
  fp.cmp_bt_stride = cmp_table_stride;
  fp.ori_rows = (int)ori_rows;
  fp.cmp_rows = (int)(scenario >= 2 ? cmp_rows : ori_rows);
  fp.ori_kv = static_cast<const uint8_t*>(ori_kv);
  fp.cmp_kv = static_cast<const uint8_t*>(scenario >= 2 ? cmp_kv : ori_kv);
  fp.ori_bt = ori_block_table;
  fp.cmp_bt = cmp_block_table;
  fp.idx = cmp_sparse_indices;
  fp.sinks = sinks;
  fp.scale_log2 = softmax_scale * kLog2e;
  fp.out = out;
  fp.lse = lse;
  fp.tok = pp.tok;
  fp.unit_start = pp.unit_start;
  fp.part_o = reinterpret_cast<float*>(ws + wl.po);
  fp.part_lse = reinterpret_cast<float*>(ws + wl.pl);
  fp.status = status;
  fp.q_box_h = q_box_h;
  fp.tau = g_tau;
  fp.trace = g_trace;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SAS_ERR_CUDA;
  static uint64_t attr_done[2] = {0, 0};  // per dtype, bit per device
  if (!(attr_done[dtype] & (1ull << dev))) {
    const cudaError_t e = dtype == SAS_DTYPE_BF16
        ? cudaFuncSetAttribute(sas_fwd_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES)
        : cudaFuncSetAttribute(sas_fwd_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return SAS_ERR_CUDA;
    attr_done[dtype] |= 1ull << dev;
  }
  if (stage_mask & SAS_STAGE_ATTENTION) {
    if (dtype == SAS_DTYPE_BF16)
      sas_fwd_kernel<0><<<R * G, kThreads, SMEM_BYTES, st>>>(tm_q, fp);
    else
      sas_fwd_kernel<1><<<R * G, kThreads, SMEM_BYTES, st>>>(tm_q, fp);
    if (cudaGetLastError() != cudaSuccess) return SAS_ERR_CUDA;
  }
  if (stage_mask & SAS_STAGE_COMBINE) {
    if (dtype == SAS_DTYPE_BF16)
      sas_combine_kernel<0><<<dim3(R, num_heads), 128, 0, st>>>(fp);
    else
      sas_combine_kernel<1><<<dim3(R, num_heads), 128, 0, st>>>(fp);
  }
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}
