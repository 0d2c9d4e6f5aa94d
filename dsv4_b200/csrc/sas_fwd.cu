// Fused sparse shared-KV attention forward for B200 (sm_100a).
//
// Two kernels, both launched by sas_sparse_attn_sharedkv_fwd on the caller's
// stream:
//
// 1. sas_plan_kernel (1 CTA): walks the metadata's per-core windows of
//    linearised (b, s) ids exactly like the reference kernel's outer loop
//    (kernel.py:254-278: pid in [bn2_start*max_seq+m_start,
//    bn2_end*max_seq+m_end), s < act_q), and gives every covered query token
//    its work in tiles: the window tile(s) plus ceil(n_cmp/512) compressed
//    tiles, n_cmp = min(K, threshold) for SCFA, threshold for CFA
//    (threshold = (s_g+1)//ratio, golden.py:41-51).
//    An exclusive scan gives each token's first unit. Output rows of
//    tokens without work are zeroed (golden.py leaves them zero), and the
//    split-token arrival counters are cleared.
//
// 2. sas_fwd_kernel (persistent, R x G CTAs, one per SM): the unit sequence
//    (one unit = one softmax tile of a token: the window rows, then the
//    compressed rows in tiles of 512, as golden.py tiles them) is cut into R
//    contiguous ranges; the G CTAs of a range each own 64 query heads (head
//    group g) and walk the same rows, so the second reader of every KV row
//    hits L2. A tile's running-max update uses that tile's exact max, so P is
//    rounded at the same points as the reference; since the max needs every
//    score of the tile first, each 128-row chunk is copied twice: K(n) for
//    the scores, then V(n) (the same rows, mostly from L2) for P.V.
//    Per CTA, warp-specialised (16 warps; warps 14-15 idle):
//      warp 3   rows: resolves window positions / top-k ids through the
//               block tables (kernel.py:285-401, 686-766) a tile at a time,
//               and publishes per chunk the pool rows, a 128-bit validity
//               mask and the chunk's flags into an 8-deep ring.
//      warps 0, 1, 12, 13 loaders: cp.async of the rows into 16 KB slabs
//               (128B-swizzled K-major; masked rows zero-filled without a
//               read), one warp instruction = 512 contiguous bytes of one
//               row, in the copy-stream order shared with the MMA thread.
//      warp 2   MMA issuer (one thread) and TMEM owner: transposed attention
//               so the KV rows fill the M=128 datapath and the 64 heads are N:
//                 S^T[128 x 64]  = K[128 x 512] . Q^T          (K-major A and B)
//                 O^T[512 x 64] += V^T[512 x 128] . P^T[128 x 64] (4 MMAs of
//               M=128; V^T is the slab pair read MN-major, since K=V)
//               TMEM: 4 score slots in cols [0,256), O^T in cols [256,512).
//      warps 4-11 softmax / epilogue, two groups of 32 heads: one thread per
//               KV row (TMEM lane). The row mask (window idx <= s_g;
//               compressed 0 <= idx < threshold, scan stopped at the first
//               -1) sets scores to -inf; per-head maxima are warp redux.max
//               plus a 4-way smem merge; the state starts at (m, l) =
//               (sink, 1) in log2 units (kernel.py:594-618, golden.py:156-160).
//               P is rounded to the I/O dtype before P.V while l sums the
//               unrounded p (golden.py:191-195). Epilogue: O/l, lse = m + ln l.
//    A token whose tiles all fall in one range is finished in place (sink
//    folded in). A token cut by range boundaries leaves normalised partials
//    (o, lse2) in the workspace; the CTA that lands the token's last partial
//    merges them: lse = log2(sum 2^lse_i + 2^sink), out = sum 2^(lse_i-lse) o_i.
//    Every wait is bounded (%globaltimer); a wait that runs out sets the
//    status word and the CTA stands down.
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
// 16 warps in 4 warpgroups. The launch gives 128 registers per thread; at the
// top of its role's branch every warp sets its limit (setmaxnreg): the
// softmax warpgroups 1-2 rise to kRegsSoftmax, warpgroups 0 and 3 drop to
// kRegsLean, which sums to the launch's 512 x 128 registers exactly.
constexpr int kMmaWarp = 2;             // warp 2: TMEM owner and MMA issuer
constexpr int kCoordWarp = 3;           // warp 3: row resolution, runs up to two tiles ahead
constexpr int kSoftmaxWarp0 = 4;        // warps 4-7: softmax group A (heads 0-31) / epilogue
constexpr int kSoftmaxWarpB = 8;        // warps 8-11: softmax group B (heads 32-63) / epilogue
constexpr int kSoftmaxWarpEnd = 12;
// warps 0, 1, 12, 13: cp.async copies of K and V rows (the sub-partitions of
// the MMA and coordinate warps hold no loader; warps 14-15 are idle)
constexpr int kLoaderWarps = 4;
constexpr int kLoaderThreads = 32 * kLoaderWarps;
constexpr int kLoaderLeadWarp = 0;
__device__ __forceinline__ bool is_loader_warp(int w) { return w < 2 || w == 12 || w == 13; }
__device__ __forceinline__ int loader_index(int w) { return w < 2 ? w : w - 10; }
constexpr int kThreads = 32 * 16;
constexpr int kRegsLaunch = 128, kRegsLean = 96, kRegsSoftmax = 160;
static_assert(256 * kRegsLean + 256 * kRegsSoftmax == kThreads * kRegsLaunch, "register split");
constexpr int kTileChunksC = 4;          // chunks per softmax tile (512 rows)
constexpr int CD = 2 * kTileChunksC;     // depth of the row-coordinate ring (chunks): two tiles
// A unit of work is one softmax tile of a token, as golden.py tiles the KV
// (GOLDEN_S2_TILE = 512 rows): the window rows, then the compressed rows in
// tiles of 512, i.e. up to kTileChunks 128-row chunks. The running max is
// updated once per tile with the tile's exact max, so P is rounded at the
// same points as the reference.
constexpr int kTileChunks = kTileChunksC;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// shared memory map (offsets from a 1024-aligned base)
// The K/V ring holds kRing 16 KB slabs. A chunk is 8 slabs; slab number n
// (counted over every chunk copy) lives in slot n % kRing. kRing is even and
// every chunk starts on an even slab number, so the slab pair (2j, 2j+1) of
// P.V's d-tile j always sits in two adjacent slots (fixed operand stride).
// The loaders copy a chunk in two halves of kSpan = 4 slabs: one warp
// instruction copies 512 contiguous bytes of one row (16 B per lane, into 4
// slabs), so a half occupies 4 consecutive slots and 8 slots keep two halves
// in flight. Measured on this B200 with 148 CTAs gathering random 1 KB rows:
// 4 rows x 128 B per instruction fill ~17 B/cycle per SM whatever the warp
// count or ring depth; 512-byte row spans from 4 warps with 8 slots, ~29.
constexpr int kSpan = 4;
constexpr int kRing = 8;
constexpr int kPBuf = 1;                                   // P^T buffers: chunk n uses buffer n % kPBuf
constexpr int P_BYTES = CH * 128;                         // one P^T buffer, 16 KB
constexpr int OFF_Q = 0;
constexpr int OFF_KV = OFF_Q + NSLAB * Q_SLAB_BYTES;     // 64 KB
constexpr int OFF_P = OFF_KV + kRing * SLAB_BYTES;       // +96 KB
constexpr int OFF_MISC = OFF_P + kPBuf * P_BYTES;
// misc region
constexpr int M_BAR = 0;         // 48 mbarriers x 8 B
constexpr int M_TMEM = 384;      // tmem base address
constexpr int M_ABORT = 392;     // sas::CtaCtl (abort flag, wait limit), 16 B
constexpr int M_LWORD = 408;     // 3 words: group B (softmax warps 8-11) OR
constexpr int M_SWORD = 420;     // 3 words: group A (softmax warps 4-7) OR
constexpr int M_RANGE = 432;     // RangeInfo of this CTA (4 ints)
constexpr int M_CMASK = 448;     // CD x 4 words: row-validity mask per ring slot
constexpr int M_RED = M_CMASK + CD * 16;  // [2 tile parities][4 quads][64 heads] per-warp maxima, 2 KB
constexpr int M_MRUN = M_RED + 2048;      // [2 groups][4 quads][32 heads] each warp's running max, 1 KB
constexpr int M_INV = M_MRUN + 1024;      // 64 floats: 1/l
constexpr int M_LRED = M_INV + 256;       // [4 quads][64 heads] per-warp row sums (epilogue), 1 KB
constexpr int M_COORD = M_LRED + 1024;    // CD x 128 int32: pool row per chunk row (-1 = masked)
constexpr int M_CINFO = M_COORD + CD * CH * 4;  // CD x int2: chunk flags and token (ChunkFlag)
constexpr int M_MW = M_CINFO + CD * 8;           // kTmemMergeMax x 64 floats: merge weights
constexpr int kTmemMergeMax = 4;                 // pieces merged straight from TMEM (else via L2)
constexpr int MISC_BYTES = M_MW + kTmemMergeMax * 64 * 4;
constexpr int kFusedMaxT = 512;  // token plans built inside the attention kernel (no plan kernel)
// fused plan region: TokInfo[kFusedMaxT], units[kFusedMaxT + 1], smax
constexpr int OFF_PLAN = OFF_MISC + MISC_BYTES;
constexpr int P_US = kFusedMaxT * 8;  // TokInfo[kFusedMaxT]
constexpr int P_SMAX = P_US + (kFusedMaxT + 1) * 4;
constexpr int PLAN_BYTES = (P_SMAX + 4 + 15) / 16 * 16;
constexpr int SMEM_BYTES = OFF_PLAN + PLAN_BYTES + 1024;  // fused plan; + alignment slack
constexpr int SMEM_BYTES_BASE = OFF_PLAN + 1024;           // plan kernel's plan: more L1 left
static_assert(SMEM_BYTES <= 232448, "shared memory over the per-CTA limit");

// barrier indices
constexpr int B_FULL = 0;        // kRing
constexpr int B_EMPTY = 8;       // kRing
constexpr int B_QFULL = 16;
constexpr int B_QEMPTY = 17;
constexpr int B_DRAIN = 18;      // the MMA thread's final commit: every tcgen05.mma it issued is done
constexpr int B_OFULL = 20;
constexpr int B_OEMPTY = 21;
// Per P^T buffer b (chunk n uses buffer n % 2), so that each completes once per
// two chunks and no waiter can fall two phases behind:
constexpr int B_PREADY2 = 32;    // 2: P^T(n) written by both softmax groups (256 arrivals)
constexpr int B_PFREE = 34;      // 2: P.V(n) done, buffer n % 2 may be rewritten
constexpr int B_CFULL = 22;      // CD: coordinate ring slot written
constexpr int B_LSYNC = 30;      // group barrier of softmax group B (warps 8-11)
constexpr int B_SSYNC = 31;      // group barrier of softmax group A (warps 4-7)
constexpr int B_CEMPTY = 36;     // CD: slot done with by the loader warps, the softmax warps and the MMA
constexpr int B_SF = 44;         // kTileChunks: S^T of chunk n landed in TMEM slot n % kTileChunks
static_assert(B_CFULL + CD <= B_LSYNC && B_CEMPTY + CD <= B_SF && B_SF + kTileChunks <= 48, "barrier map");
constexpr int kCemptyCount = kLoaderWarps + 8 + 1;  // loader warps + softmax warps + the MMA thread
// P^T buffer of chunk n, and the phase parity of that buffer's barriers for it
__device__ __forceinline__ uint32_t pbuf(uint32_t n) { return n % kPBuf; }
__device__ __forceinline__ uint32_t pphase(uint32_t n) { return (n / kPBuf) & 1; }

// Per-chunk flags published by the coordinate warp with the chunk's rows
// (int2 {flags, token} per coordinate-ring slot).
enum ChunkFlag : int {
  CF_END = 1,         // no chunk: the stream has ended
  CF_WIN = 2,         // window chunk (ori pool), else compressed
  CF_SEG_FIRST = 4,   // first chunk of a segment
  CF_SEG_LAST = 8,    // last chunk of a segment
  CF_TILE_LAST = 16,  // last chunk of a softmax tile
};

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t TM_S = 0;     // S^T: kTileChunks slots of 64 columns, chunk n in slot n % kTileChunks
constexpr uint32_t TM_O = 256;   // O^T: 4 d-tiles of 64 columns

// A query token: its request and causal end position s_g. Its compressed
// threshold and row count follow from s_g (tok_thr / tok_ncmp).
struct TokInfo {
  int b, s_g;
};
static_assert(sizeof(TokInfo) == 8, "fused plan layout");

// Outputs of the head-sharded multi-GPU forward (the GA kernel variants): the
// call computes heads [h0, h0 + H) of outputs holding H_total heads per
// token and writes every result into the output buffers of all n ranks
// (peer pointers into symmetric memory), so the outputs are gathered as they
// are produced and no all-gather follows. Lives in the workspace.
constexpr int kMaxOut = 8;
struct OutDesc {
  uint8_t* out[kMaxOut];
  float* lse[kMaxOut];  // lse[0] == nullptr: no LSE
  int n, H_total, h0;
  __device__ __forceinline__ size_t row(int t, int hh) const { return (size_t)t * H_total + h0 + hh; }
  __device__ __forceinline__ void st32(int t, int hh, int col, uint32_t w) const {
    const size_t off = (row(t, hh) * D + col) * 2;
    for (int k = 0; k < n; ++k) *reinterpret_cast<uint32_t*>(out[k] + off) = w;
  }
  __device__ __forceinline__ void st64(int t, int hh, int col, uint2 w) const {
    const size_t off = (row(t, hh) * D + col) * 2;
    for (int k = 0; k < n; ++k) *reinterpret_cast<uint2*>(out[k] + off) = w;
  }
  __device__ __forceinline__ void st16(int t, int hh, int col, uint16_t w) const {
    const size_t off = (row(t, hh) * D + col) * 2;
    for (int k = 0; k < n; ++k) *reinterpret_cast<uint16_t*>(out[k] + off) = w;
  }
  __device__ __forceinline__ void lse_st(int t, int hh, float v) const {
    if (lse[0])
      for (int k = 0; k < n; ++k) lse[k][row(t, hh)] = v;
  }
  // zero the H heads of token t, threads [i0, i0 + stride) of the caller
  __device__ __forceinline__ void zero_token(int t, int H, int i0, int stride) const {
    for (int k = 0; k < n; ++k) {
      uint4* o = reinterpret_cast<uint4*>(out[k] + row(t, 0) * D * 2);
      for (int i = i0; i < H * D * 2 / 16; i += stride) o[i] = make_uint4(0, 0, 0, 0);
      if (lse[0])
        for (int h = i0; h < H; h += stride) lse[k][row(t, h)] = 0.f;
    }
  }
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
  int32_t* merge_cnt;   // [n_cnt] split-token arrival counters, zeroed here
  int n_cnt;
  const OutDesc* god;   // head-sharded outputs (nullptr: out / lse above)
};

struct FwdParams {
  int T, H, G, R, scenario, K, ratio, win_left, n_win_chunks;
  int ori_bs, ori_bt_stride, cmp_bs, cmp_bt_stride;
  int ori_nblk, cmp_nblk;  // pool sizes in blocks: table entries outside [0, nblk) are dropped and flagged
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
  int32_t* merge_cnt;  // [R*G*2]: arrivals per cut token, keyed by (first range, group, head half)
  int32_t* status;
  int q_box_h;
  float tau;                 // lazy-rescale threshold, log2 units (0 = exact running max)
  int cut_cost;              // split tokens longer than a range plus this many tiles (< 0: never)
  unsigned long long wait_ns;  // limit of every bounded wait
  // fused plan (T <= kFusedMaxT): the CTA builds the token plan itself and
  // checks metadata coverage at output time
  int fused, early;          // early: the preceding kernel is our metadata kernel
  int B, S, layout;
  const int32_t* cu;
  const int32_t* seqused_kv;
  const int32_t* meta;
  unsigned long long* trace; // optional per-CTA cycle counters (nullptr in production)
  const OutDesc* god;        // head-sharded outputs, read by the GA kernel variants only
};

// trace slots per CTA (SM cycles, accumulated by one thread of each role)
enum TraceSlot {
  TR_TOTAL = 0, TR_P_COORD, TR_P_WAIT_EMPTY, TR_P_WAIT_MASK, TR_P_ISSUE, TR_M_WAIT_Q, TR_M_WAIT_FULL,
  TR_M_WAIT_P, TR_M_WAIT_O, TR_S_WAIT_MASK, TR_S_WAIT_S, TR_S_SOFTMAX, TR_S_WAIT_O, TR_S_EPI, TR_CHUNKS,
  TR_SEGS, TR_E_TMEM, TR_E_STAGE, TR_E_COPY, TR_E_RED, TR_S_LD, TR_S_SYNC1, TR_S_SYNC2, TR_S_EXP,
  TR_S_SUM, TR_S_FENCE, TR_S_RESCALE, TR_S_MAX, TR_FIRST_S, TR_PROLOGUE, TR_NSLOTS = 30
};

// Tiles of a token: ceil(window chunks / 4) window tiles, then the
// compressed chunks in groups of 4 (golden.py walks ori tiles, then cmp tiles).
__device__ __forceinline__ int token_tiles(int n_win_chunks, int n_cmp) {
  return (n_win_chunks + kTileChunks - 1) / kTileChunks + ((n_cmp + CH - 1) / CH + kTileChunks - 1) / kTileChunks;
}
// Chunk range [c0, c1) of tile k (chunk c < n_win_chunks is a window chunk,
// else compressed chunk c - n_win_chunks).
__device__ __forceinline__ void tile_chunks(int k, int n_win_chunks, int n_cmp, int& c0, int& c1) {
  const int nwt = (n_win_chunks + kTileChunks - 1) / kTileChunks;
  if (k < nwt) {
    c0 = k * kTileChunks;
    c1 = min(c0 + kTileChunks, n_win_chunks);
  } else {
    const int ncc = (n_cmp + CH - 1) / CH;
    c0 = n_win_chunks + (k - nwt) * kTileChunks;
    c1 = n_win_chunks + min((k - nwt + 1) * kTileChunks, ncc);
  }
}

__device__ __forceinline__ int py_floordiv(int a, int b) {
  int q = a / b, r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) --q;
  return q;
}
// threshold = (s_g + 1) // ratio: compressed ids at or past it are masked
// (golden.py:41-51); the rows a token scans: min(K, threshold) top-k slots
// for SCFA, every compressed row below the threshold for CFA, none for SWA
__device__ __forceinline__ int tok_thr(int s_g, int scenario, int ratio) {
  return scenario == 1 ? 0 : max(py_floordiv(s_g + 1, ratio), 0);
}
__device__ __forceinline__ int tok_ncmp(int thr, int scenario, int K) {
  return scenario == 3 ? min(K, thr) : (scenario == 2 ? thr : 0);
}

// ------------------------------------------------------------------ plan
__global__ void __launch_bounds__(1024, 1) sas_plan_kernel(PlanParams p) {
  sas::pdl_launch_dependents();  // the attention kernel's prologue may start now
  sas::pdl_wait();               // the metadata may come from the kernel before
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
  for (int i = tid; i < p.n_cnt; i += blockDim.x) p.merge_cnt[i] = 0;
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
      TokInfo ti{b, 0};
      if (s < act_q && b < p.B) {
        const int pid = b * smax + s;
        bool covered = false;
        for (int i = 0; i < SAS_AIC_CORE_NUM; ++i)
          covered |= (s_en[i] != 0) && pid >= s_lin[i][0] && pid < s_lin[i][1];
        const int act_kv = p.seqused_kv[b];
        const int s_g = act_kv - act_q + s;
        const int n_cmp = tok_ncmp(tok_thr(s_g, p.scenario, p.ratio), p.scenario, p.K);
        ti.s_g = s_g;
        if (covered) units = token_tiles(p.n_win_chunks, n_cmp);
      }
      p.tok[t] = ti;
      if (units == 0) {
        // padding / uncovered token: zero output and LSE (golden.py leaves them zero)
        if (p.god) {
          p.god->zero_token(t, p.H, 0, 1);
        } else {
          uint4* o = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + (size_t)t * p.H * D * p.dtype_bytes);
          for (int i = 0; i < p.H * D * p.dtype_bytes / 16; ++i) o[i] = make_uint4(0, 0, 0, 0);
          if (p.lse)
            for (int h = 0; h < p.H; ++h) p.lse[(size_t)t * p.H + h] = 0.f;
        }
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

// Largest t in [0, T) with us[t] <= x (us non-decreasing, us[0] <= x),
// found by one warp in 32-way steps: ceil(log32 T) rounds of loads instead of
// log2 T dependent ones. Every lane returns the result.
__device__ __forceinline__ int warp_last_le(const int32_t* us, int T, int x, int lane) {
  int lo = 0, hi = T - 1;
  while (hi > lo) {
    const int step = (hi - lo + 32) / 32;  // probes lo + k*step, k = 1..32, cover (lo, hi]
    const int probe = lo + (lane + 1) * step;
    const bool le = probe <= hi && us[probe] <= x;
    const unsigned b = __ballot_sync(0xffffffffu, le);
    if (b == 0) {
      hi = lo + step - 1;
    } else {
      const int k = 31 - __clz(b);  // last probe with us[probe] <= x
      lo = lo + (k + 1) * step;
      hi = min(hi, lo + step - 1);
    }
  }
  return lo;
}

// First unit of range r: r*u, moved back to the start of the token holding
// it unless splitting is enabled (cut_cost >= 0) and the token holds more
// than a range plus cut_cost tiles; boundaries inside a split token are
// therefore always r*u exactly. By default tokens are never split: the
// reference keeps every token on one core, and a piece that starts a token's
// softmax from the sink rounds P against its own running max, not the token's.
__device__ __forceinline__ int range_start(const int32_t* us, int T, int U, int u, int r, int lane, int cut_cost) {
  if (r <= 0) return 0;
  const long long x = (long long)r * u;
  if (x >= U) return U;
  const int t = warp_last_le(us, T, (int)x, lane);
  const int st = us[t], n = us[t + 1] - st;
  return (x == st || (cut_cost >= 0 && n > u + cut_cost)) ? (int)x : st;
}

// A CTA's unit range [u0, end) and the token holding u0, computed once per
// CTA by one warp and shared through shared memory.
struct RangeInfo {
  int u0, end, t, u;
};

__device__ __forceinline__ RangeInfo compute_range(const int32_t* us, int T, int R, int r, int lane, int cut_cost) {
  RangeInfo ri;
  const int U = us[T];
  ri.u = (U + R - 1) / R;
  ri.u0 = range_start(us, T, U, ri.u, r, lane, cut_cost);
  ri.end = r + 1 >= R ? U : range_start(us, T, U, ri.u, r + 1, lane, cut_cost);
  ri.t = ri.u0 < U ? warp_last_le(us, T, ri.u0, lane) : T - 1;
  return ri;
}

struct Walker {
  int pos, end, t, u0, u;
  const int32_t* us;
  __device__ void init(const int32_t* unit_start, const RangeInfo& ri) {
    us = unit_start;
    u = ri.u;
    u0 = ri.u0;
    pos = u0;
    end = ri.end;
    t = ri.t;
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

// One tile of this CTA's work in stream order (tiles of consecutive segments).
struct Tile {
  int t, c0, nch;
  uint32_t seg, g0;  // segment number; global number of the tile's first chunk
  bool first, last;  // first / last tile of its segment
};

// Walks this CTA's tiles across segment boundaries, so that the copy and MMA
// roles can look one tile ahead.
struct TileIter {
  Walker wk;
  Seg sg;
  int k, n_cmp;
  uint32_t seg, g;
  bool started;
  __device__ void init(const int32_t* unit_start, const RangeInfo& ri) {
    wk.init(unit_start, ri);
    started = false;
    seg = 0;
    g = 0;
    k = 0;
    sg.ce = 0;
  }
  __device__ bool next(Tile& tl, const TokInfo* tokp, int n_win_chunks, int scenario, int ratio, int K) {
    if (!started || k >= sg.ce) {
      if (!wk.next(sg)) return false;
      if (started) ++seg;
      started = true;
      k = sg.cb;
      n_cmp = tok_ncmp(tok_thr(tokp[sg.t].s_g, scenario, ratio), scenario, K);
    }
    int c1;
    tile_chunks(k, n_win_chunks, n_cmp, tl.c0, c1);
    tl.t = sg.t;
    tl.nch = c1 - tl.c0;
    tl.seg = seg;
    tl.g0 = g;
    tl.first = k == sg.cb;
    tl.last = k == sg.ce - 1;
    g += tl.nch;
    ++k;
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
  __device__ static T zero() { return __float2bfloat16_rn(0.f); }
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
  __device__ static T zero() { return __float2half_rn(0.f); }
};

// Reduce 64 per-thread values across the 32 lanes of a warp; afterwards
// v[0], v[1] hold the reduction for columns 2*lane and 2*lane+1.
// Warp reduce-scatter of N = 32 or 64 per-lane columns: afterwards lane l
// holds the reduction over the 32 lanes for columns [l*N/32, (l+1)*N/32) in
// v[0 .. N/32). Five exchange rounds, each halving the live columns.
template <int N, bool IS_MAX>
__device__ __forceinline__ void warp_reduce_scatter(float (&v)[N], int lane) {
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    const int half = (N / 2) >> step;
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

__device__ __forceinline__ bool twait(uint64_t* bar, uint32_t parity, volatile sas::CtaCtl* abort_flag, int* status,
                                      int where, bool tracing, unsigned long long& acc) {
  const long long t0 = tracing ? clock64() : 0;
  const bool r = sas::mbar_wait(bar, parity, abort_flag, status, where);
  if (tracing) acc += clock64() - t0;
  return r;
}

// The order in which the loaders copy, and the MMA issuer consumes, the two
// passes over every chunk n: K(n), the rows for S^T = K Q^T, and V(n), the
// same rows again for O^T += V^T P^T. Both roles step this rule in lockstep
// (it depends only on the chunk flags the coordinate warp publishes):
//  - K(n) as soon as n <= nv + 4: S^T(n) goes to TMEM slot n % 4, free once
//    the exp pass of chunk n - 4 has read it, and that exp pass needs only
//    stream items before K(n) (the S^T of its tile, P.V of chunks n - 6 and
//    n - 5);
//  - else V(nv), which needs the tile's max, i.e. every K of its tile.
// The scores of the next tiles are therefore computed while P.V of the
// current one runs, across token boundaries.
enum StreamItem { SI_K = 0, SI_V = 1, SI_END = 2, SI_FAIL = 3 };
struct Stream {
  uint32_t nk = 0, nv = 0;  // next chunk for K, for V
  bool kend = false;        // every chunk has had its K
  template <bool TR>
  __device__ __forceinline__ int next(uint64_t* bars, const int2* cinfo, volatile sas::CtaCtl* abort_flag, int* status,
                                      unsigned long long& tslot) {
    if (!kend && nk <= nv + kTileChunks) {
      if (!twait(&bars[B_CFULL + nk % CD], (nk / CD) & 1, abort_flag, status, 3, TR, tslot)) return SI_FAIL;
      if (!(cinfo[nk % CD].x & CF_END)) return SI_K;
      kend = true;
    }
    if (nv == nk) return SI_END;  // only once kend: else K(nk) was taken above
    if (kend) return SI_V;
    for (uint32_t j = nv; j < nk; ++j)
      if (cinfo[j % CD].x & CF_TILE_LAST) return SI_V;
    return SI_FAIL;  // unreachable: nk > nv + 4 spans a whole tile
  }
};

// Barrier among the 4 warps of one role, with a bounded wait (a named
// barrier cannot time out, and a sibling warp that left on an abort would
// strand the others in it). Lane 0 of every warp arrives on `bar` (count 4);
// `pred` is OR-reduced into words[ph % 3]; warp `lead` clears the word the
// sync after next uses before it arrives: every warp has read that word
// (two syncs back) before it arrived at the previous sync. Returns false
// when the wait gave up.
struct GroupSync {
  uint64_t* bar;
  uint32_t* words;
  uint32_t ph;
  __device__ __forceinline__ bool sync_or(int pred, int lane, bool lead, int& result, volatile sas::CtaCtl* abort_flag,
                                          int* status, int where) {
    const bool any = __any_sync(0xffffffffu, pred);
    __syncwarp();
    const uint32_t k = ph % 3;
    if (lane == 0) {
      if (any) atomicOr(&words[k], 1u);
      if (lead) words[(k + 1) % 3] = 0;
      sas::mbar_arrive(bar);
    }
    const bool ok = sas::mbar_wait(bar, ph & 1, abort_flag, status, where);
    result = ok ? (int)*reinterpret_cast<volatile uint32_t*>(&words[k]) : 0;
    ++ph;
    return ok;
  }
  __device__ __forceinline__ bool sync(int lane, bool lead, volatile sas::CtaCtl* abort_flag, int* status, int where) {
    int unused;
    return sync_or(0, lane, lead, unused, abort_flag, status, where);
  }
};

// 16-byte async copy global -> shared; src_bytes = 0 writes zeros without reading.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// Arrive on `bar` once every cp.async issued so far by this thread has landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(sas::smem_u32(bar)) : "memory");
}

// One softmax group: 4 warps that cover TMEM lanes 0-127 (one KV row of the
// chunk per thread) and 32 of the CTA's 64 heads, S^T / O^T columns
// [hb, hb+32). Group A is warps 4-7 (hb = 0); group B is the loader warps
// 0-3 (hb = 32), which are otherwise idle while the chunk they copied is in
// softmax. The groups own disjoint heads, so they never wait on each other.
struct SmGroup {
  int hb, half;         // first head column (0 or 32), hb / 32
  int quad, lane, gst;  // TMEM lane quadrant, lane, row = quad*32 + lane
  bool lead;
  GroupSync gs;
  float lsum[32];       // running sums of heads hb..hb+31 over this thread's row
                        // (reduced over the 128 rows once per segment)
  uint32_t lane_addr;   // TMEM address of this warp's lane quadrant
  uint32_t seg;         // segments finished
};

// Shared-memory scratch of the softmax groups (disjoint columns per group).
struct SmShared {
  float* red;     // [2 chunk parities][4 quads][64 heads] per-warp maxima
  float* m_run;   // [2 groups][4 quads][32 heads]: each warp's own copy of the running max
  float* inv;     // [64] 1 / l
  float* lred;    // [4 quads][64 heads] per-warp row sums of a segment
  uint8_t* pbuf;  // P^T: 128 rows x 64 heads, 128B-swizzled
  float* scratch; // [kTmemMergeMax][64]: merge weights / LSEs
};

// This warp's running max for its group's 32 heads.
__device__ __forceinline__ float* warp_mrun(const SmShared& S, const SmGroup& G) {
  return S.m_run + (G.half * 4 + G.quad) * 32;
}

// The token plan this CTA uses (from the 1024-aligned shared-memory base
// that the barriers sit in): its own fused plan, or the plan kernel's.
__device__ __forceinline__ const uint8_t* smem_base_of(const uint64_t* bars) {
  return reinterpret_cast<const uint8_t*>(bars) - M_BAR - OFF_MISC;
}

// Split-KV merge of one cut token for the heads [hb, hb+32) of group g, run
// by one softmax group of the CTA that wrote the token's last partial:
// lse = log2(sum_i 2^lse_i + 2^sink), out = sum_i 2^(lse_i - lse) o_i.
// Phase 1: thread c folds head hb+c's partial LSEs in one online pass.
// Phase 2: every thread owns one float4 column and accumulates 8 heads at a
// time, so 8 independent loads are in flight per partial. Partials come
// from other CTAs, so they are read through L2 (.cg).
// Workspace slot of range rr's partial of a cut token whose first range is r0;
// wf = 1 when that token is not the first segment of range r0.
__device__ __forceinline__ size_t part_slot(const FwdParams& p, int rr, int r0, int wf, int g) {
  return ((size_t)rr * 2 + (rr == r0 ? wf : 0)) * p.G + g;
}

template <int DT, bool GA>
__device__ __forceinline__ bool merge_cut_token(const FwdParams& p, int t, int g, int r0, int r1, int wf,
                                                SmGroup& G, float* lse_s, volatile sas::CtaCtl* abort_flag) {
  using IO = IoType<DT>;
  const int ns = r1 - r0 + 1;
  const int hn = min(HG, p.H - g * HG);  // heads of this group
  const int hend = min(G.hb + 32, hn);
  if (G.hb + G.gst < hend && G.gst < 32) {
    const int c = G.hb + G.gst, h = g * HG + c;
    float m = p.sinks[h] * kLog2e, den = 1.f;
    for (int i = 0; i < ns; ++i) {
      const float l = __ldcg(p.part_lse + part_slot(p, r0 + i, r0, wf, g) * HG + c);
      const float mn = fmaxf(m, l);
      den = den * sas::ex2(m - mn) + sas::ex2(l - mn);
      m = mn;
    }
    const float L = m + __log2f(den);
    lse_s[c] = L;
    if constexpr (GA) p.god->lse_st(t, h, L * kLn2);
    else if (p.lse) p.lse[(size_t)t * p.H + h] = L * kLn2;
  }
  if (!G.gs.sync(G.lane, G.lead, abort_flag, p.status, 22)) return false;
  typename IO::T* outp = reinterpret_cast<typename IO::T*>(p.out) + ((size_t)t * p.H + g * HG) * D;
  constexpr int kHB = 8;
#pragma unroll 1
  for (int h0 = G.hb; h0 < hend; h0 += kHB) {
    float4 acc[kHB];
#pragma unroll
    for (int j = 0; j < kHB; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
    for (int i = 0; i < ns; ++i) {
      const size_t slot = part_slot(p, r0 + i, r0, wf, g);
      const float* pl = p.part_lse + slot * HG + h0;
      const float4* po = reinterpret_cast<const float4*>(p.part_o + (slot * HG + h0) * D) + G.gst;
      float4 v[kHB];
      float w[kHB];
#pragma unroll
      for (int j = 0; j < kHB; ++j) {
        v[j] = __ldcg(po + j * (D / 4));
        w[j] = __ldcg(pl + j);
      }
#pragma unroll
      for (int j = 0; j < kHB; ++j) {
        const float wj = sas::ex2(w[j] - lse_s[h0 + j]);
        acc[j].x += wj * v[j].x;
        acc[j].y += wj * v[j].y;
        acc[j].z += wj * v[j].z;
        acc[j].w += wj * v[j].w;
      }
    }
#pragma unroll
    for (int j = 0; j < kHB; ++j) {
      if (h0 + j < hend) {
        uint2 o;
        o.x = IO::pack(acc[j].x, acc[j].y);
        o.y = IO::pack(acc[j].z, acc[j].w);
        if constexpr (GA) p.god->st64(t, g * HG + h0 + j, 4 * G.gst, o);
        else reinterpret_cast<uint2*>(outp + (size_t)(h0 + j) * D)[G.gst] = o;
      }
    }
  }
  return true;
}

// Max pass over one tile for the group's 32 heads (golden.py:187-190): the
// per-head max of the tile's scores (masked rows excluded) over the 128 rows
// of every chunk, merged over the 4 quads; the running max m becomes
// max(m, tile max). Every warp merges the quads' maxima itself and keeps its
// own copy of m, so one group barrier suffices; the maxima are double-buffered
// by tile parity. al / need: the rescale factor 2^(m_old - m_new) of this
// thread's lane head, and whether any head's max moved.
template <int DT>
__device__ __forceinline__ bool tile_max_pass(const FwdParams& p, SmGroup& G, const SmShared& S, uint64_t* bars,
                                              const uint32_t* cmask, uint32_t gtile, uint32_t gch0, int nch,
                                              bool first_tile_of_seg, int g, float& al, int& need,
                                              volatile sas::CtaCtl* abort_flag, bool tracing, unsigned long long* tr) {
  float* mw = warp_mrun(S, G);
  if (first_tile_of_seg) {
    const int h = g * HG + G.hb + G.lane;
    mw[G.lane] = h < p.H ? p.sinks[h] * kLog2e : 0.f;  // (m, l) start at (sink, 1): golden.py:162-163
#pragma unroll
    for (int h2 = 0; h2 < 32; ++h2) G.lsum[h2] = 0.f;
  }
  long long ts0 = 0;
  float mx[32];
#pragma unroll
  for (int h = 0; h < 32; ++h) mx[h] = -INFINITY;
#pragma unroll 1
  for (int i = 0; i < nch; ++i) {
    const uint32_t n = gch0 + i;
    if (!twait(&bars[B_SF + n % kTileChunks], (n / kTileChunks) & 1, abort_flag, p.status, 9, tracing,
               tr[TR_S_WAIT_S]))
      return false;
    sas::tc_fence_after();
    if (tracing && i == 0) ts0 = clock64();
    const bool valid = (cmask[(n % CD) * 4 + G.quad] >> G.lane) & 1;
    uint32_t ra[32];
    sas::tmem_ld32(G.lane_addr + TM_S + 64 * (n % kTileChunks) + G.hb, ra);
    sas::tmem_wait_ld();
    if (valid) {
#pragma unroll
      for (int h = 0; h < 32; ++h) mx[h] = fmaxf(mx[h], __uint_as_float(ra[h]) * p.scale_log2);
    }
  }
#pragma unroll
  for (int h = 0; h < 32; h += 4) {
    float4 w;
    w.x = sas::warp_max_f32(mx[h]);
    w.y = sas::warp_max_f32(mx[h + 1]);
    w.z = sas::warp_max_f32(mx[h + 2]);
    w.w = sas::warp_max_f32(mx[h + 3]);
    if (G.lane == 0) *reinterpret_cast<float4*>(S.red + (gtile & 1) * 256 + G.quad * 64 + G.hb + h) = w;
  }
  if (!G.gs.sync(G.lane, G.lead, abort_flag, p.status, 16)) return false;
  {
    const float* rb = S.red + (gtile & 1) * 256 + G.hb + G.lane;
    const float tmx = fmaxf(fmaxf(rb[0], rb[64]), fmaxf(rb[128], rb[192]));
    const float mo = mw[G.lane];
    const bool up = tmx > mo + p.tau;
    al = 1.f;
    if (up) {
      al = sas::ex2(mo - tmx);
      mw[G.lane] = tmx;
    }
    need = __any_sync(0xffffffffu, up);
    __syncwarp();
  }
  if (tracing) tr[TR_S_MAX] += clock64() - ts0;
  return true;
}

// Exp pass of one chunk of the tile: p = 2^(x - m) with the tile's m (masked
// rows give 0), rounded to the I/O dtype into P^T, l += sum of the unrounded
// p (golden.py:191-195). The first chunk of a tile applies the tile's rescale
// to l and O^T (golden.py:192,196) once the previous P.V is done.
template <int DT>
__device__ __forceinline__ bool chunk_exp_pass(const FwdParams& p, SmGroup& G, const SmShared& S, uint64_t* bars,
                                               const uint32_t* cmask, uint32_t gchunk, int i, bool rescale_now,
                                               bool first_tile_of_seg, float al, uint32_t& gp,
                                               volatile sas::CtaCtl* abort_flag, bool tracing, unsigned long long* tr) {
  using IO = IoType<DT>;
  const long long ts0 = tracing ? clock64() : 0;
  const float* mw = warp_mrun(S, G);
  const bool valid = (cmask[(gchunk % CD) * 4 + G.quad] >> G.lane) & 1;
  float x[32];
  {
    uint32_t ra[32];
    sas::tmem_ld32(G.lane_addr + TM_S + 64 * (gchunk % kTileChunks) + G.hb, ra);
    sas::tmem_wait_ld();
#pragma unroll
    for (int h = 0; h < 32; ++h) x[h] = valid ? sas::ex2(__uint_as_float(ra[h]) * p.scale_log2 - mw[h]) : 0.f;
  }
  // P buffer pbuf(gp) is free once P.V of chunk gp - kPBuf is done; a
  // rescale of O^T also needs P.V of chunk gp - 1 done
  if (gp >= (uint32_t)kPBuf && !twait(&bars[B_PFREE + pbuf(gp - kPBuf)], pphase(gp - kPBuf), abort_flag, p.status,
                                      13, tracing, tr[TR_S_WAIT_O]))
    return false;
  if (kPBuf > 1 && rescale_now && gp > 0 &&
      !twait(&bars[B_PFREE + pbuf(gp - 1)], pphase(gp - 1), abort_flag, p.status, 13, tracing, tr[TR_S_WAIT_O]))
    return false;
  sas::tc_fence_after();
  if (rescale_now) {
#pragma unroll
    for (int h = 0; h < 32; ++h) G.lsum[h] *= __shfl_sync(0xffffffffu, al, h);
    if (!first_tile_of_seg) {
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {
        uint32_t o[32];
        sas::tmem_ld32(G.lane_addr + TM_O + 64 * j + G.hb, o);
        sas::tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 32; ++h)
          o[h] = __float_as_uint(__uint_as_float(o[h]) * __shfl_sync(0xffffffffu, al, h));
        sas::tmem_st32(G.lane_addr + TM_O + 64 * j + G.hb, o);
      }
      sas::tmem_wait_st();
    }
  }
#pragma unroll
  for (int h = 0; h < 32; ++h) G.lsum[h] += x[h];
  uint8_t* prow = S.pbuf + pbuf(gp) * P_BYTES + G.gst * 128;
#pragma unroll
  for (int c4 = 0; c4 < 4; ++c4) {
    const int cc = (G.hb >> 3) + c4;  // 16-byte column chunk of the 128-byte row
    const int h = c4 * 8;
    *reinterpret_cast<uint4*>(prow + ((cc ^ (G.gst & 7)) << 4)) =
        make_uint4(IO::pack(x[h], x[h + 1]), IO::pack(x[h + 2], x[h + 3]), IO::pack(x[h + 4], x[h + 5]),
                   IO::pack(x[h + 6], x[h + 7]));
  }
  sas::fence_proxy_async_smem();
  sas::tc_fence_before();
  sas::mbar_arrive(&bars[B_PREADY2 + pbuf(gp)]);
  ++gp;
  if (tracing) {
    tr[TR_S_SOFTMAX] += clock64() - ts0;
    tr[TR_CHUNKS] += 1;
  }
  return true;
}

// Merge of a cut token for the group's heads, run by the piece that lands
// last, with its own piece straight from TMEM: the other pieces' normalised
// partials (o_i, lse_i) are read through L2, its own is O/l in registers,
// bit-identical to the partial it would have written. Every piece enters the
// same way in range order, so the result does not depend on which piece
// merges: lse = log2(2^sink + sum_i 2^lse_i), out = sum_i 2^(lse_i - lse) o_i.
template <int DT, bool GA>
__device__ __forceinline__ bool merge_from_tmem(const FwdParams& p, SmGroup& G, const SmShared& S, float* mw,
                                                int t, int g, int r0, int r1, int wf, int own_r,
                                                volatile sas::CtaCtl* abort_flag) {
  using IO = IoType<DT>;
  const int np = r1 - r0 + 1;  // <= kTmemMergeMax
  if (G.gst < 32) {
    const int c = G.hb + G.gst, h = g * HG + c;
    const float L = S.lred[c] + S.lred[64 + c] + S.lred[128 + c] + S.lred[192 + c];
    const float own = L > 0.f ? warp_mrun(S, G)[G.gst] + __log2f(L) : -INFINITY;  // as the partial's lse
    const float sink = h < p.H ? p.sinks[h] * kLog2e : 0.f;
    float li[kTmemMergeMax];
    float M = sink;
    for (int i = 0; i < np; ++i) {
      const int rr = r0 + i;
      li[i] = rr == own_r ? own : __ldcg(p.part_lse + part_slot(p, rr, r0, wf, g) * HG + c);
      M = fmaxf(M, li[i]);
    }
    float den = sas::ex2(sink - M);
    for (int i = 0; i < np; ++i) den += sas::ex2(li[i] - M);
    const float lse = M + __log2f(den);
    for (int i = 0; i < np; ++i) mw[i * 64 + c] = sas::ex2(li[i] - lse);
    if constexpr (GA) {
      if (h < p.H) p.god->lse_st(t, h, lse * kLn2);
    } else if (p.lse && h < p.H) {
      p.lse[(size_t)t * p.H + h] = lse * kLn2;
    }
  }
  if (!G.gs.sync(G.lane, G.lead, abort_flag, p.status, 23)) return false;
  typename IO::T* outp = reinterpret_cast<typename IO::T*>(p.out) + (size_t)t * p.H * D;
  const int row = G.gst;
  const bool odd = G.lane & 1;
  const int d_even = row & ~1;
  // 16 heads per pass keeps the accumulators, the loads and the own O^T
  // values within the register budget of the epilogue
#pragma unroll 1
  for (int pass = 0; pass < 8; ++pass) {
    const int j = pass >> 1, hs = (pass & 1) * 16;  // O^T tile, first head of the pass
    float acc[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) acc[h] = 0.f;
#pragma unroll 1
    for (int i = 0; i < np; ++i) {
      const int rr = r0 + i;
      float v[16];
      if (rr == own_r) {
        uint32_t o[16];
        sas::tmem_ld16(G.lane_addr + TM_O + 64 * j + G.hb + hs, o);
        sas::tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 16; ++h) v[h] = __fmul_rn(__uint_as_float(o[h]), S.inv[G.hb + hs + h]);  // as written
      } else {
        const float* src =
            p.part_o + part_slot(p, rr, r0, wf, g) * HG * D + (size_t)(G.hb + hs) * D + j * 128 + row;
#pragma unroll
        for (int h = 0; h < 16; ++h) v[h] = __ldcg(src + (size_t)h * D);
      }
#pragma unroll
      for (int h = 0; h < 16; ++h) acc[h] = __fmaf_rn(mw[i * 64 + G.hb + hs + h], v[h], acc[h]);
    }
    // lanes pair up (row, row^1): the even lane stores heads hs..hs+7, the odd one hs+8..hs+15
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      const float recv = __shfl_xor_sync(0xffffffffu, odd ? acc[h] : acc[h + 8], 1);
      const uint32_t w = odd ? IO::pack(recv, acc[h + 8]) : IO::pack(acc[h], recv);
      const int hh = g * HG + G.hb + hs + (odd ? h + 8 : h);
      if constexpr (GA) {
        if (hh < p.H) p.god->st32(t, hh, j * 128 + d_even, w);
      } else if (hh < p.H) {
        *reinterpret_cast<uint32_t*>(outp + (size_t)hh * D + j * 128 + d_even) = w;
      }
    }
  }
  return true;
}

// Epilogue of one segment for the group's heads: l over the 4 quads, then
// out = O/l with the sink folded into l (complete token), or, for a token cut
// across CTAs, the split-KV protocol: every piece but the last to finish
// leaves a normalised partial (o, lse2); the last merges them. If all other
// pieces are already in when a CTA gets here, it merges from its own TMEM and
// never writes its partial.
template <int DT, bool GA>
__device__ __forceinline__ bool segment_epilogue(const FwdParams& p, SmGroup& G, const SmShared& S, uint64_t* bars,
                                                 const Seg& sg, int r, int g, volatile sas::CtaCtl* abort_flag, bool tracing,
                                                 unsigned long long* tr) {
  using IO = IoType<DT>;
  if (!twait(&bars[B_OFULL], G.seg & 1, abort_flag, p.status, 10, tracing, tr[TR_S_WAIT_O])) return false;
  sas::tc_fence_after();
  const long long te0 = tracing ? clock64() : 0;
  {
    // the segment's l: this warp's 32 rows, then the 4 quads through smem
    float l[32];
#pragma unroll
    for (int h = 0; h < 32; ++h) l[h] = G.lsum[h];
    warp_reduce_scatter<32, false>(l, G.lane);
    S.lred[G.quad * 64 + G.hb + G.lane] = l[0];
  }
  if (!G.gs.sync(G.lane, G.lead, abort_flag, p.status, 18)) return false;

  const size_t pslot = ((size_t)r * 2 + sg.which) * p.G + g;
  if (G.gst < 32) {
    const int c = G.hb + G.gst, h = g * HG + c;
    const float L = S.lred[c] + S.lred[64 + c] + S.lred[128 + c] + S.lred[192 + c];
    const float m = warp_mrun(S, G)[G.gst];  // threads 0-31 are the quad-0 warp
    if (sg.complete) {
      const float sink = h < p.H ? p.sinks[h] * kLog2e : 0.f;
      const float Lf = L + sas::ex2(sink - m);
      S.inv[c] = 1.f / Lf;
      if constexpr (GA) {
        if (h < p.H) p.god->lse_st(sg.t, h, (m + __log2f(Lf)) * kLn2);
      } else if (p.lse && h < p.H) {
        p.lse[(size_t)sg.t * p.H + h] = (m + __log2f(Lf)) * kLn2;
      }
    } else {
      S.inv[c] = L > 0.f ? 1.f / L : 0.f;
    }
  }
  // the ranges holding the token's pieces: r0 .. r1 (wf: r0 holds an earlier token first)
  int r0 = r, r1 = r, wf = 0;
  int32_t* cnt = nullptr;
  int early = 0;
  if (!sg.complete) {
    const RangeInfo ri = *reinterpret_cast<const RangeInfo*>(reinterpret_cast<uint8_t*>(bars) - M_BAR + M_RANGE);
    const int32_t* us = p.fused ? reinterpret_cast<const int32_t*>(smem_base_of(bars) + OFF_PLAN + P_US)
                                : p.unit_start;
    const int ust = us[sg.t], un = us[sg.t + 1] - ust;
    r0 = ust / ri.u;
    r1 = (ust + un - 1) / ri.u;
    wf = r0 * ri.u < ust ? 1 : 0;
    cnt = p.merge_cnt + ((size_t)r0 * p.G + g) * 2 + G.half;
    if (G.gst == 0 && r1 - r0 < kTmemMergeMax) early = atomicAdd(cnt, 0) == r1 - r0;
  }
  if (!G.gs.sync_or(early, G.lane, G.lead, early, abort_flag, p.status, 19)) return false;
  if (tracing) tr[TR_E_RED] += clock64() - te0;
  const int row = G.gst;  // d within an O^T tile
  if (sg.complete) {
    // direct stores: lanes pair up (row, row^1); the even lane stores head h
    // for both rows, the odd lane head h+16 (4-byte stores; no shared-memory
    // staging, which would compete with the MMA operand reads)
    typename IO::T* outp = reinterpret_cast<typename IO::T*>(p.out) + (size_t)sg.t * p.H * D;
    const bool odd = G.lane & 1;
    const int d_even = row & ~1;
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      uint32_t o[32];
      sas::tmem_ld32(G.lane_addr + TM_O + 64 * j + G.hb, o);
      sas::tmem_wait_ld();
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float v0 = __uint_as_float(o[h]) * S.inv[G.hb + h];
        const float v1 = __uint_as_float(o[h + 16]) * S.inv[G.hb + h + 16];
        const float recv = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 1);
        const uint32_t w = odd ? IO::pack(recv, v1) : IO::pack(v0, recv);
        const int hh = g * HG + G.hb + (odd ? h + 16 : h);
        if constexpr (GA) {
          if (hh < p.H) p.god->st32(sg.t, hh, j * 128 + d_even, w);
        } else if (hh < p.H) {
          *reinterpret_cast<uint32_t*>(outp + (size_t)hh * D + j * 128 + d_even) = w;
        }
      }
    }
  } else {
    int tmem_merge = early;
    if (early) {
      // every other piece is in: reset the counter for the next launch
      if (G.gst == 0) *cnt = 0;
    } else {
    if (G.gst < 32) {
      const int c = G.hb + G.gst;
      const float L = S.lred[c] + S.lred[64 + c] + S.lred[128 + c] + S.lred[192 + c];
      p.part_lse[pslot * HG + c] = L > 0.f ? warp_mrun(S, G)[G.gst] + __log2f(L) : -INFINITY;
    }
    float* po = p.part_o + pslot * HG * D;
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      uint32_t o[32];
      sas::tmem_ld32(G.lane_addr + TM_O + 64 * j + G.hb, o);
      sas::tmem_wait_ld();
#pragma unroll
      for (int h = 0; h < 32; ++h)
        po[(size_t)(G.hb + h) * D + j * 128 + row] = __fmul_rn(__uint_as_float(o[h]), S.inv[G.hb + h]);
    }
    // every piece adds one arrival (per head half) to the counter of the
    // token's first range; the one that lands last merges
    __threadfence();
    if (!G.gs.sync(G.lane, G.lead, abort_flag, p.status, 20)) return false;
    int mine = 0, is_last = 0;
    if (G.gst == 0) {
      mine = atomicAdd(cnt, 1) == r1 - r0;
      if (mine) *cnt = 0;  // every arrival is in: reset for the next launch
    }
    if (!G.gs.sync_or(mine, G.lane, G.lead, is_last, abort_flag, p.status, 21)) return false;
    if (is_last) {
      if (r1 - r0 < kTmemMergeMax) {
        tmem_merge = 1;
      } else {
        __threadfence();
        if (!merge_cut_token<DT, GA>(p, sg.t, g, r0, r1, wf, G, S.scratch, abort_flag)) return false;
      }
    }
    }
    if (tmem_merge) {
      __threadfence();
      float* mw = S.scratch;
      if (!merge_from_tmem<DT, GA>(p, G, S, mw, sg.t, g, r0, r1, wf, r, abort_flag)) return false;
    }
  }
  sas::tc_fence_before();
  sas::mbar_arrive(&bars[B_OEMPTY]);
  ++G.seg;
  if (tracing) {
    tr[TR_S_EPI] += clock64() - te0;
    tr[TR_SEGS] += 1;
  }
  return true;
}

// A complete token's epilogue in two halves, so that the softmax groups can
// start the next token's first tile in between (its max pass and first exp
// pass overlap the last P.V of this token):
//  - first half, before the next tile: l over the 4 quads, 1/l with the sink
//    folded in, lse (golden.py:201-205); needs only this thread's sums and
//    the running max, not O^T;
//  - second half, after it: O^T / l from TMEM to the output rows, then O^T is
//    released to the MMA.
// The next tile's max pass holds a group barrier, which orders the first
// half's shared-memory writes before the second half's reads.
template <int DT, bool GA>
__device__ __forceinline__ bool epilogue_first_half(const FwdParams& p, SmGroup& G, const SmShared& S, const Seg& sg,
                                                    int g, volatile sas::CtaCtl* abort_flag) {
  float l[32];
#pragma unroll
  for (int h = 0; h < 32; ++h) l[h] = G.lsum[h];
  warp_reduce_scatter<32, false>(l, G.lane);
  S.lred[G.quad * 64 + G.hb + G.lane] = l[0];
  if (!G.gs.sync(G.lane, G.lead, abort_flag, p.status, 18)) return false;
  if (G.gst < 32) {
    const int c = G.hb + G.gst, h = g * HG + c;
    const float L = S.lred[c] + S.lred[64 + c] + S.lred[128 + c] + S.lred[192 + c];
    const float m = warp_mrun(S, G)[G.gst];  // threads 0-31 are the quad-0 warp
    const float sink = h < p.H ? p.sinks[h] * kLog2e : 0.f;
    const float Lf = L + sas::ex2(sink - m);
    S.inv[c] = 1.f / Lf;
    if constexpr (GA) {
      if (h < p.H) p.god->lse_st(sg.t, h, (m + __log2f(Lf)) * kLn2);
    } else if (p.lse && h < p.H) {
      p.lse[(size_t)sg.t * p.H + h] = (m + __log2f(Lf)) * kLn2;
    }
  }
  return true;
}

template <int DT, bool GA>
__device__ __forceinline__ bool epilogue_second_half(const FwdParams& p, SmGroup& G, const SmShared& S,
                                                     uint64_t* bars, const Seg& sg, int g, volatile sas::CtaCtl* abort_flag,
                                                     bool tracing, unsigned long long* tr) {
  using IO = IoType<DT>;
  if (!twait(&bars[B_OFULL], G.seg & 1, abort_flag, p.status, 10, tracing, tr[TR_S_WAIT_O])) return false;
  sas::tc_fence_after();
  const long long te0 = tracing ? clock64() : 0;
  // direct stores: lanes pair up (row, row^1); the even lane stores head h
  // for both rows, the odd lane head h+16
  const int row = G.gst;  // d within an O^T tile
  typename IO::T* outp = reinterpret_cast<typename IO::T*>(p.out) + (size_t)sg.t * p.H * D;
  const bool odd = G.lane & 1;
  const int d_even = row & ~1;
#pragma unroll 1
  for (int j = 0; j < 4; ++j) {
    uint32_t o[32];
    sas::tmem_ld32(G.lane_addr + TM_O + 64 * j + G.hb, o);
    sas::tmem_wait_ld();
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      const float v0 = __uint_as_float(o[h]) * S.inv[G.hb + h];
      const float v1 = __uint_as_float(o[h + 16]) * S.inv[G.hb + h + 16];
      const float recv = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 1);
      const uint32_t w = odd ? IO::pack(recv, v1) : IO::pack(v0, recv);
      const int hh = g * HG + G.hb + (odd ? h + 16 : h);
      if constexpr (GA) {
        if (hh < p.H) p.god->st32(sg.t, hh, j * 128 + d_even, w);
      } else if (hh < p.H) {
        *reinterpret_cast<uint32_t*>(outp + (size_t)hh * D + j * 128 + d_even) = w;
      }
    }
  }
  sas::tc_fence_before();
  sas::mbar_arrive(&bars[B_OEMPTY]);
  ++G.seg;
  if (tracing) {
    tr[TR_S_EPI] += clock64() - te0;
    tr[TR_SEGS] += 1;
  }
  return true;
}

// Fused plan: metadata coverage (kernel.py:254-278 windows) is checked after
// the fact. Every token with work was written as if covered; once the
// metadata is complete, each softmax group walks its range again and zeroes
// its heads of every token that no core window covers (the reference leaves
// those zero). The piece that merges a cut token does this after its merge,
// so an uncovered cut token ends zero whatever the order of the pieces.
template <int DT, bool GA>
__device__ bool zero_uncovered(const FwdParams& p, SmGroup& G, const int32_t* us, const TokInfo* tok,
                               const int* s_smax, const RangeInfo& ri, int g, volatile sas::CtaCtl* abort_flag) {
  using IO = IoType<DT>;
  sas::pdl_wait();  // the metadata is complete and visible
  const int smax = *s_smax;
  int lin0 = 0, lin1 = 0;  // this thread's core window, if any
  if (G.gst < SAS_AIC_CORE_NUM) {
    const int32_t* row = p.meta + G.gst * 8;
    if (row[0] != 0) {
      lin0 = row[1] * smax + row[2];
      lin1 = row[4] * smax + row[5];
    }
  }
  Walker wk;
  wk.init(us, ri);
  Seg sg;
  while (wk.next(sg)) {
    const int b = tok[sg.t].b;
    const int q = b * smax + (sg.t - (p.layout == SAS_LAYOUT_TND ? p.cu[b] : b * p.S));  // pid of kernel.py
    int covered;
    if (!G.gs.sync_or(q >= lin0 && q < lin1, G.lane, G.lead, covered, abort_flag, p.status, 24)) return false;
    if (covered) continue;
    typename IO::T* outp = reinterpret_cast<typename IO::T*>(p.out) + (size_t)sg.t * p.H * D;
    for (int h = 0; h < 32; ++h) {
      const int hh = g * HG + G.hb + h;
      if (hh < p.H)
        for (int j = 0; j < 4; ++j) {
          if constexpr (GA) p.god->st16(sg.t, hh, j * 128 + G.gst, 0);
          else outp[(size_t)hh * D + j * 128 + G.gst] = IO::zero();
        }
    }
    if constexpr (GA) {
      if (G.gst < 32 && g * HG + G.hb + G.gst < p.H) p.god->lse_st(sg.t, g * HG + G.hb + G.gst, 0.f);
    } else if (p.lse && G.gst < 32 && g * HG + G.hb + G.gst < p.H) {
      p.lse[(size_t)sg.t * p.H + g * HG + G.hb + G.gst] = 0.f;
    }
  }
  return true;
}

// The plan kernel's work for up to kFusedMaxT tokens, done by every CTA of
// the attention kernel into its own shared memory: per-token info and the
// exclusive scan of chunk units. Metadata coverage is not applied here (the
// epilogue checks it before writing a token), so none of this reads the
// metadata and it can run while the metadata kernel is still in flight.
// Output rows of tokens without work are zeroed, each by one CTA.
template <int DT, bool GA>
__device__ void fused_plan(const FwdParams& p, TokInfo* s_tok, int32_t* s_us, int* s_smax, int* s_wsum) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kW = kThreads / 32;
  // max_seq: the reference api's S_max (api.py:208-215 / 229)
  int mx = 0;
  if (p.layout == SAS_LAYOUT_TND) {
    // seqused_kv is loaded in this first pass too (into L1), so the per-request
    // pass below finds both arrays there: one cold round trip, not two
    int kv = 0;
    for (int b = tid; b < p.B; b += kThreads) {
      mx = max(mx, p.cu[b + 1] - p.cu[b]);
      kv |= p.seqused_kv[b];
    }
    if (kv == -1) mx = max(mx, 0);  // keeps the loads; never true for valid lengths
  } else {
    mx = p.S;
  }
  for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_wsum[warp] = mx;
  __syncthreads();
  int smax = 0;
  for (int w = 0; w < kW; ++w) smax = max(smax, s_wsum[w]);
  // one thread per request (TND) or per token (BSND): no per-token search
  auto plan_token = [&](int t, int b, int s, int act_q) {
    TokInfo ti{b, 0};
    int units = 0;
    if (s < act_q && b < p.B) {
      const int s_g = p.seqused_kv[b] - act_q + s;
      ti.s_g = s_g;
      units = token_tiles(p.n_win_chunks, tok_ncmp(tok_thr(s_g, p.scenario, p.ratio), p.scenario, p.K));
    }
    s_tok[t] = ti;
    s_us[t] = units;
  };
  if (p.layout == SAS_LAYOUT_TND) {
    for (int b = tid; b < p.B; b += kThreads) {
      const int c0 = p.cu[b], c1 = min(p.cu[b + 1], p.T);
      for (int t = c0; t < c1; ++t) plan_token(t, b, t - c0, c1 - c0);
    }
    // tokens past cu[B] (none for a well-formed batch) carry no work
    for (int t = p.cu[p.B] + tid; t < p.T; t += kThreads) plan_token(t, p.B, 0, 0);
  } else {
    for (int t = tid; t < p.T; t += kThreads) {
      const int b = t / p.S, s = t - b * p.S;
      plan_token(t, b, s, p.cu ? p.cu[b + 1] - p.cu[b] : p.S);
    }
  }
  __syncthreads();
  // tokens without work keep zero output and LSE (golden.py leaves them zero)
  for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
    if (s_us[t] != 0) continue;
    if constexpr (GA) {
      p.god->zero_token(t, p.H, tid, kThreads);
    } else {
      uint4* o = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + (size_t)t * p.H * D * 2);
      for (int i = tid; i < p.H * D * 2 / 16; i += kThreads) o[i] = make_uint4(0, 0, 0, 0);
      if (p.lse)
        for (int h = tid; h < p.H; h += kThreads) p.lse[(size_t)t * p.H + h] = 0.f;
    }
  }
  // exclusive scan of the units, in place: each thread a run of <= 2 tokens
  constexpr int kPer = (kFusedMaxT + kThreads - 1) / kThreads;
  const int b0 = tid * kPer;
  int v[kPer];
  int local = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    v[i] = b0 + i < p.T ? s_us[b0 + i] : 0;
    local += v[i];
  }
  int incl = local;
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  __syncthreads();
  if (lane == 31) s_wsum[warp] = incl;
  __syncthreads();
  int run = incl - local;
  for (int w = 0; w < warp; ++w) run += s_wsum[w];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    if (b0 + i < p.T) s_us[b0 + i] = run;
    run += v[i];
  }
  if (tid == kThreads - 1) s_us[p.T] = run;  // the total
  if (tid == 0) *s_smax = smax;
  __syncthreads();
}

// TRACE = true builds the diagnostics variant that accumulates per-role cycle
// counters into p.trace; the production variant carries none of that state.
template <int DT, bool TRACE, bool FUSED, bool GA>
__global__ void __launch_bounds__(kThreads, 1)
    sas_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const FwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const long long t_entry = TRACE ? clock64() : 0;
  const uint32_t raw_addr = sas::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  uint8_t* misc = smem + OFF_MISC;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + M_BAR);
  volatile sas::CtaCtl* abort_flag = reinterpret_cast<volatile sas::CtaCtl*>(misc + M_ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + M_TMEM);
  uint32_t* cmask = reinterpret_cast<uint32_t*>(misc + M_CMASK);        // [CD][4]
  int32_t* coords = reinterpret_cast<int32_t*>(misc + M_COORD);          // [CD][128]
  int2* cinfo = reinterpret_cast<int2*>(misc + M_CINFO);                 // [CD] {ChunkFlag bits, token}
  float* red = reinterpret_cast<float*>(misc + M_RED);
  float* m_run = reinterpret_cast<float*>(misc + M_MRUN);
  float* inv_s = reinterpret_cast<float*>(misc + M_INV);
  // the token plan: this CTA's own (FUSED) or the plan kernel's
  TokInfo* s_tok = reinterpret_cast<TokInfo*>(smem + OFF_PLAN);
  int32_t* s_us = reinterpret_cast<int32_t*>(smem + OFF_PLAN + P_US);
  const int32_t* usp = FUSED ? s_us : p.unit_start;
  const TokInfo* tokp = FUSED ? s_tok : p.tok;
  const SmShared sm{red, m_run, inv_s, reinterpret_cast<float*>(misc + M_LRED), smem + OFF_P,
                    reinterpret_cast<float*>(misc + M_MW)};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = blockIdx.x / p.G, g = blockIdx.x % p.G;

  if (tid == 0) {
    for (int i = 0; i < kRing; ++i) {
      sas::mbar_init(&bars[B_FULL + i], kLoaderThreads);
      sas::mbar_init(&bars[B_EMPTY + i], 1);
    }
    sas::mbar_init(&bars[B_QFULL], 1);
    sas::mbar_init(&bars[B_QEMPTY], 1);
    sas::mbar_init(&bars[B_DRAIN], 1);
    for (int i = 0; i < kTileChunks; ++i) sas::mbar_init(&bars[B_SF + i], 1);
    sas::mbar_init(&bars[B_OFULL], 1);
    sas::mbar_init(&bars[B_OEMPTY], 256);
    for (int i = 0; i < kPBuf; ++i) {
      sas::mbar_init(&bars[B_PREADY2 + i], 256);
      sas::mbar_init(&bars[B_PFREE + i], 1);
    }
    for (int i = 0; i < CD; ++i) {
      sas::mbar_init(&bars[B_CFULL + i], 1);
      sas::mbar_init(&bars[B_CEMPTY + i], kCemptyCount);
    }
    sas::mbar_init(&bars[B_SSYNC], 4);
    sas::mbar_init(&bars[B_LSYNC], 4);
    for (int i = 0; i < 3; ++i) {
      reinterpret_cast<uint32_t*>(misc + M_SWORD)[i] = 0;
      reinterpret_cast<uint32_t*>(misc + M_LWORD)[i] = 0;
    }
    abort_flag->abort = 0;
    abort_flag->limit_ns = p.wait_ns;
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
  // everything above overlaps the kernel before; in early mode (fused plan,
  // the kernel before is our metadata kernel, which writes nothing read here)
  // the metadata is only waited for when a token's output is written
  if (!p.early) sas::pdl_wait();
  if constexpr (FUSED)
    fused_plan<DT, GA>(p, s_tok, s_us,
                   reinterpret_cast<int*>(smem + OFF_PLAN + P_SMAX), reinterpret_cast<int*>(red));
  if (warp == 0) {
    const RangeInfo ri = compute_range(usp, p.T, p.R, r, lane, p.cut_cost);
    if (lane == 0) *reinterpret_cast<RangeInfo*>(misc + M_RANGE) = ri;
  }
  if (tid == 32) sas::tma_prefetch_desc(&tm_q);
  sas::tc_fence_before();
  __syncthreads();
  sas::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr bool tracing = TRACE;
  unsigned long long tr[TR_NSLOTS];
#pragma unroll
  for (int i = 0; i < TR_NSLOTS; ++i) tr[i] = 0;
  const long long t_start = tracing ? clock64() : 0;
  // event timeline of the CTA's first chunks (trace builds only): slot i of
  // 16 per CTA after the counters, SM cycles since kernel entry
  auto ev = [&](int i) {
    if (TRACE) p.trace[(size_t)gridDim.x * TR_NSLOTS + (size_t)blockIdx.x * 16 + i] = clock64() - t_entry;
  };
  if (TRACE && tid == 0) ev(15);

  // Register split: each role sets its limit at the top of its branch, so the
  // compiler allocates every branch under that limit; all warps of a
  // warpgroup execute the same value (warps 0-3 and 12-15: kRegsLean, warps
  // 4-11: kRegsSoftmax).
  if (warp == kCoordWarp) {
    sas::setmaxnreg_dec<kRegsLean>();
    // =============================== row resolution, up to CD chunks ahead
    // Lane l resolves rows l, l+32, l+64, l+96 of every chunk through the
    // block tables (kernel.py:285-401, 686-766) and writes the pool row (or
    // -1) and the validity mask into the ring.
    // A whole tile (up to 4 chunks) is resolved per round with all its loads
    // in flight together: the index rows, then the block-table entries.
    TileIter it;
    it.init(usp, *reinterpret_cast<const RangeInfo*>(misc + M_RANGE));
    Tile tl;
    TokInfo ti{};
    int ti_thr = 0, ti_ncmp = 0;
    bool stopped = false, ok = true;
    while (ok && it.next(tl, tokp, p.n_win_chunks, p.scenario, p.ratio, p.K)) {
      const long long tc0 = tracing ? clock64() : 0;
      if (tl.first) {
        ti = tokp[tl.t];
        ti_thr = tok_thr(ti.s_g, p.scenario, p.ratio);
        ti_ncmp = tok_ncmp(ti_thr, p.scenario, p.K);
        // the compressed scan stops at the first -1 (golden.py:55-56): a range
        // that starts inside a token looks for one in the slots before it
        stopped = false;
        const int cmp_c0 = max(tl.c0 - p.n_win_chunks, 0);
        if (p.scenario == 3 && cmp_c0 > 0) {
          const int lim = min(cmp_c0 * CH, ti_ncmp);
          const int32_t* ip = p.idx + (size_t)tl.t * p.K;
          int neg = 0;
          for (int e = lane; e < lim; e += 32) neg |= (ip[e] == -1);
          stopped = __any_sync(0xffffffffu, neg);
        }
      }
      const bool is_win = tl.c0 < p.n_win_chunks;  // a tile is all window or all compressed
      int coord[kTileChunks][4];
      bool val[kTileChunks][4];
      // a block-table column past the table's width (a seqused_kv longer than
      // the table) or an entry past the pool is dropped like a -1 entry, and
      // reported (non-fatal) in the status word
      bool bad = false;
      if (is_win) {
        const int lo = max(ti.s_g - p.win_left, 0);
#pragma unroll
        for (int j = 0; j < kTileChunks; ++j)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int pos = lo + (tl.c0 + j) * CH + k * 32 + lane;
            val[j][k] = j < tl.nch && ti.s_g >= 0 && pos <= ti.s_g;
            const int col = pos / p.ori_bs;
            const bool in_table = col < p.ori_bt_stride;
            const int blk = val[j][k] && in_table ? p.ori_bt[(size_t)ti.b * p.ori_bt_stride + col] : -1;
            bad |= val[j][k] && (!in_table || blk >= p.ori_nblk);
            val[j][k] = val[j][k] && blk >= 0 && blk < p.ori_nblk;
            coord[j][k] = blk * p.ori_bs + pos % p.ori_bs;
          }
      } else {
        const int e0 = (tl.c0 - p.n_win_chunks) * CH;
#pragma unroll
        for (int j = 0; j < kTileChunks; ++j)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int e = e0 + j * CH + k * 32 + lane;
            val[j][k] = j < tl.nch && e < ti_ncmp;
            coord[j][k] = e;  // the compressed id, until resolved
            if (p.scenario == 3) coord[j][k] = val[j][k] ? p.idx[(size_t)tl.t * p.K + e] : 0;
          }
        if (p.scenario == 3) {
#pragma unroll
          for (int j = 0; j < kTileChunks; ++j) {
            int cf = CH;  // first -1 of this chunk, in row order
#pragma unroll
            for (int k = 3; k >= 0; --k) {
              const unsigned bal = __ballot_sync(0xffffffffu, val[j][k] && coord[j][k] == -1);
              if (bal) cf = k * 32 + __ffs(bal) - 1;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k)
              val[j][k] = val[j][k] && !stopped && k * 32 + lane < cf && coord[j][k] >= 0 && coord[j][k] < ti_thr;
            stopped = stopped || (j < tl.nch && cf < CH);
          }
        } else {
#pragma unroll
          for (int j = 0; j < kTileChunks; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k) val[j][k] = val[j][k] && coord[j][k] < ti_thr;
        }
#pragma unroll
        for (int j = 0; j < kTileChunks; ++j)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int id = coord[j][k];
            const int col = id / p.cmp_bs;
            const bool in_table = col < p.cmp_bt_stride;
            const int blk = val[j][k] && in_table ? p.cmp_bt[(size_t)ti.b * p.cmp_bt_stride + col] : -1;
            bad |= val[j][k] && (!in_table || blk >= p.cmp_nblk);
            val[j][k] = val[j][k] && blk >= 0 && blk < p.cmp_nblk;
            coord[j][k] = val[j][k] ? blk * p.cmp_bs + id % p.cmp_bs : 0;
          }
      }
      if (__any_sync(0xffffffffu, bad) && lane == 0 && p.status) atomicCAS(p.status, 0, SAS_ERR_BAD_BLOCK_ENTRY);
      if (tracing) tr[TR_P_COORD] += clock64() - tc0;
      if (TRACE && lane == 0 && tl.g0 == 0) ev(0);
      if (TRACE && lane == 0 && tl.g0 > 0 && tl.g0 <= (uint32_t)kTileChunks && !tl.first) ev(2);
#pragma unroll
      for (int j = 0; j < kTileChunks; ++j) {
        if (j >= tl.nch) break;
        const uint32_t gc = tl.g0 + j;
        const int slot = gc % CD;
        if (!twait(&bars[B_CEMPTY + slot], ((gc / CD) & 1) ^ 1, abort_flag, p.status, 2, tracing,
                   tr[TR_P_WAIT_MASK])) {
          ok = false;
          break;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          coords[slot * CH + k * 32 + lane] = val[j][k] ? coord[j][k] : -1;
          const unsigned vb = __ballot_sync(0xffffffffu, val[j][k]);
          if (lane == 0) cmask[slot * 4 + k] = vb;
        }
        if (lane == 0) {
          const int fl = (is_win ? CF_WIN : 0) | (tl.first && j == 0 ? CF_SEG_FIRST : 0) |
                         (tl.last && j == tl.nch - 1 ? CF_SEG_LAST : 0) | (j == tl.nch - 1 ? CF_TILE_LAST : 0);
          cinfo[slot] = make_int2(fl, tl.t);
        }
        __syncwarp();
        if (lane == 0) sas::mbar_arrive(&bars[B_CFULL + slot]);
        if (TRACE && lane == 0 && gc == 0) ev(1);
        if (TRACE && lane == 0 && gc == 4) ev(3);
      }
    }
    if (ok) {  // the end of the stream, as one more ring slot
      const uint32_t gc = it.g;
      const int slot = gc % CD;
      if (twait(&bars[B_CEMPTY + slot], ((gc / CD) & 1) ^ 1, abort_flag, p.status, 2, tracing, tr[TR_P_WAIT_MASK])) {
        if (lane == 0) {
          cinfo[slot] = make_int2(CF_END, 0);
          sas::mbar_arrive(&bars[B_CFULL + slot]);
        }
      }
    }
  } else if (is_loader_warp(warp)) {
    sas::setmaxnreg_dec<kRegsLean>();
    // =============================== loaders: K rows, then V rows, per tile
    // The copies run in the MMA's consumption order (K of every chunk of a
    // tile, then V of every chunk) and block only on ring slots, which QK^T
    // and P.V free as they read them.
    const int lw = loader_index(warp);  // rows [32*lw, 32*lw+32) of every chunk
    const int sl = lane >> 3, c16 = lane & 7;  // slab of the half, 16-byte piece of its 128 bytes
    const bool lead = tid == kLoaderLeadWarp * 32;
    const uint32_t kv_base = sas::smem_u32(smem + OFF_KV);
    uint32_t sc = 0;  // ring slabs filled so far
    const uint32_t q_bytes = (uint32_t)NSLAB * p.q_box_h * 128;
    bool ok = true;
    // copy the 128 rows of chunk-slot `cslot` (pool rows resolved by the
    // coordinate warp) into the ring, in two halves of kSpan slabs:
    // instruction i of a half copies 512 contiguous bytes of row 32*lw + i,
    // lane l the 16 B piece c16 of slab sl; every lane then arrives on the
    // half's slab barriers
    auto load_chunk = [&](uint32_t cslot, bool is_win) -> bool {
      const int myrow = coords[cslot * CH + lw * 32 + lane];  // lane i holds row 32*lw + i
      const uint8_t* pool = is_win ? p.ori_kv : p.cmp_kv;
      for (int h = 0; h < NSLAB / kSpan; ++h, sc += kSpan) {
#pragma unroll
        for (int j = 0; j < kSpan; ++j)
          if (!twait(&bars[B_EMPTY + (sc + j) % kRing], (((sc + j) / kRing) & 1) ^ 1, abort_flag, p.status, 3,
                     tracing, tr[TR_P_WAIT_EMPTY]))
            return false;
        const uint32_t slab = kv_base + ((sc + sl) % kRing) * SLAB_BYTES;
        const uint8_t* src0 = pool + (h * kSpan + sl) * 128 + c16 * 16;
#pragma unroll 8
        for (int i = 0; i < 32; ++i) {
          const int row = __shfl_sync(0xffffffffu, myrow, i);
          const int rl = lw * 32 + i;
          const bool v = row >= 0;
          cp_async16(slab + rl * 128 + ((c16 ^ (rl & 7)) << 4), src0 + (size_t)(v ? row : 0) * (D * 2), v ? 16u : 0u);
        }
#pragma unroll
        for (int j = 0; j < kSpan; ++j) cp_async_arrive(&bars[B_FULL + (sc + j) % kRing]);
      }
      return true;
    };
    Stream st;
    uint32_t seg_i = 0, q_loads = 0;
    while (ok) {
      const int item = st.next<tracing>(bars, cinfo, abort_flag, p.status, tr[TR_P_WAIT_MASK]);
      if (item == SI_END) break;
      if (item == SI_FAIL) {
        ok = false;
        break;
      }
      if (item == SI_K) {
        const uint32_t n = st.nk++;
        const int2 ci = cinfo[n % CD];
        if (ci.x & CF_SEG_FIRST) {
          if (lead) {
            if (!twait(&bars[B_QEMPTY], (seg_i & 1) ^ 1, abort_flag, p.status, 1, tracing, tr[TR_P_WAIT_EMPTY])) {
              ok = false;
            } else {
              sas::mbar_arrive_expect_tx(&bars[B_QFULL], q_bytes);
              for (int s = 0; s < NSLAB; ++s)
                sas::tma_load_3d(smem + OFF_Q + s * Q_SLAB_BYTES, &tm_q, &bars[B_QFULL], s * 64, g * HG, ci.y);
              ++q_loads;
            }
          }
          ++seg_i;
        }
        if (ok) ok = load_chunk(n % CD, ci.x & CF_WIN);
        if (TRACE && lead && n == 0) ev(5);
        if (TRACE && lead && n == 4) ev(6);
      } else {  // V rows: the K rows again, mostly from L2
        const uint32_t n = st.nv++;
        ok = load_chunk(n % CD, cinfo[n % CD].x & CF_WIN);
        if (TRACE && lead && n == 0) ev(4);
        __syncwarp();
        if (lane == 0) sas::mbar_arrive(&bars[B_CEMPTY + n % CD]);
      }
    }
    // nothing may still be landing in shared memory when the CTA exits (an
    // aborted CTA leaves the loop with copies in flight)
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (lead && q_loads > 0) sas::mbar_wait_drain(&bars[B_QFULL], (q_loads - 1) & 1, SAS_WAIT_LIMIT_NS);
  } else if (warp == kMmaWarp) {
    sas::setmaxnreg_dec<kRegsLean>();
    // =============================== MMA issuer
    // Per tile: S^T of every chunk into its own TMEM slot as the K rows land,
    // then, per chunk, O^T += V^T P^T as the V rows land and P is ready.
    if (lane == 0) {
      constexpr uint32_t idesc1 = sas::umma_idesc_f16(DT == 0 ? 1 : 0, 128, HG, 0, 0);
      constexpr uint32_t idesc2 = sas::umma_idesc_f16(DT == 0 ? 1 : 0, 128, HG, 1, 1);
      const uint32_t q_base = sas::smem_u32(smem + OFF_Q);
      const uint32_t kv_base = sas::smem_u32(smem + OFF_KV);
      const uint32_t p_base = sas::smem_u32(smem + OFF_P);
      Stream st;
      uint32_t sc = 0;               // ring slabs consumed so far, in the loaders' order
      uint32_t kseg = 0, vseg = 0;   // segments begun by K, by V
      bool ok = true;
      while (ok) {
        const int item = st.next<tracing>(bars, cinfo, abort_flag, p.status, tr[TR_M_WAIT_FULL]);
        if (item == SI_END || item == SI_FAIL) break;
        if (item == SI_K) {
          // ---- S^T(n) = K(n) . Q^T into TMEM slot n % 4
          const long long tq0 = tracing ? clock64() : 0;
          const uint32_t n = st.nk++;
          const int fl = cinfo[n % CD].x;
          if (fl & CF_SEG_FIRST) {
            if (!twait(&bars[B_QFULL], kseg & 1, abort_flag, p.status, 4, tracing, tr[TR_M_WAIT_Q])) break;
            ++kseg;
          }
          // the slot's previous chunk n - 4 must have been read by its exp
          // pass: implied by P.V(n - 4) if that was issued, else wait for P(n - 4)
          if (n >= (uint32_t)kTileChunks && n - kTileChunks >= st.nv &&
              !twait(&bars[B_PREADY2 + pbuf(n - kTileChunks)], pphase(n - kTileChunks), abort_flag, p.status, 6, tracing,
                     tr[TR_M_WAIT_P]))
            break;
          sas::tc_fence_after();
          const uint32_t sd = TM_S + 64 * (n % kTileChunks);
          for (int s = 0; s < NSLAB; ++s, ++sc) {
            const uint32_t slot = sc % kRing;
            if (!twait(&bars[B_FULL + slot], (sc / kRing) & 1, abort_flag, p.status, 5, tracing,
                       tr[TR_M_WAIT_FULL])) {
              ok = false;
              break;
            }
            const long long tf0 = tracing ? clock64() : 0;
            sas::fence_proxy_async_smem();  // cp.async (generic proxy) writes -> tensor-core reads
            sas::tc_fence_after();
            const long long tf1 = tracing ? clock64() : 0;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sas::umma_desc_sw128(kv_base + slot * SLAB_BYTES + kk * 32, 16, 1024);
              const uint64_t bd = sas::umma_desc_sw128(q_base + s * Q_SLAB_BYTES + kk * 32, 16, 1024);
              sas::umma_ss(tmem + sd, ad, bd, idesc1, (s | kk) != 0);
            }
            sas::umma_commit(&bars[B_EMPTY + slot]);
            if (tracing) {
              tr[TR_S_SYNC1] += tf1 - tf0;
              tr[TR_S_SYNC2] += clock64() - tf1;
            }
          }
          if (!ok) break;
          sas::umma_commit(&bars[B_SF + n % kTileChunks]);
          if (fl & CF_SEG_LAST) sas::umma_commit(&bars[B_QEMPTY]);
          if (TRACE && n == 0) ev(7);
          if (TRACE && n == 4) ev(8);
          if (tracing) tr[TR_M_WAIT_O] += clock64() - tq0;  // QK^T section, waits included
        } else {
          // ---- O^T += V^T(n) . P^T(n)
          const long long tv0 = tracing ? clock64() : 0;
          const uint32_t n = st.nv++;
          const int fl = cinfo[n % CD].x;
          const bool first = fl & CF_SEG_FIRST;
          if (!twait(&bars[B_PREADY2 + pbuf(n)], pphase(n), abort_flag, p.status, 6, tracing, tr[TR_M_WAIT_P]))
            break;
          if (first) {
            if (vseg > 0 &&
                !twait(&bars[B_OEMPTY], (vseg - 1) & 1, abort_flag, p.status, 7, tracing, tr[TR_M_WAIT_Q]))
              break;
            ++vseg;
          }
          sas::tc_fence_after();
          const uint32_t pb = p_base + pbuf(n) * P_BYTES;
          for (int j = 0; j < 4; ++j, sc += 2) {
            const uint32_t slot = sc % kRing;  // even: the pair (slot, slot + 1) never wraps
            const uint32_t par = (sc / kRing) & 1;
            if (!twait(&bars[B_FULL + slot], par, abort_flag, p.status, 12, tracing, tr[TR_M_WAIT_FULL]) ||
                !twait(&bars[B_FULL + slot + 1], par, abort_flag, p.status, 12, tracing, tr[TR_M_WAIT_FULL])) {
              ok = false;
              break;
            }
            const long long tf0 = tracing ? clock64() : 0;
            sas::fence_proxy_async_smem();
            sas::tc_fence_after();
            if (tracing) tr[TR_S_SYNC1] += clock64() - tf0;
            const long long tf1 = tracing ? clock64() : 0;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t ad = sas::umma_desc_sw128(kv_base + slot * SLAB_BYTES + kk * 2048, SLAB_BYTES, 1024);
              const uint64_t bd = sas::umma_desc_sw128(pb + kk * 2048, 8192, 1024);
              sas::umma_ss(tmem + TM_O + 64 * j, ad, bd, idesc2, (first && kk == 0) ? 0u : 1u);
            }
            sas::umma_commit(&bars[B_EMPTY + slot]);
            sas::umma_commit(&bars[B_EMPTY + slot + 1]);
            if (tracing) tr[TR_S_EXP] += clock64() - tf1;
          }
          if (!ok) break;
          sas::umma_commit(&bars[B_PFREE + pbuf(n)]);
          if (fl & CF_SEG_LAST) sas::umma_commit(&bars[B_OFULL]);
          sas::mbar_arrive(&bars[B_CEMPTY + n % CD]);  // done with the chunk's flags
          if (TRACE && n == 0) ev(9);
          if (TRACE && n == 4) ev(10);
          if (tracing) tr[TR_E_COPY] += clock64() - tv0;  // P.V section, waits included
        }
      }
      // every MMA issued must be done before TMEM is freed (an aborted CTA
      // leaves the loop with MMAs in flight)
      sas::umma_commit(&bars[B_DRAIN]);
      sas::mbar_wait_drain(&bars[B_DRAIN], 0, SAS_WAIT_LIMIT_NS);
    }
    __syncwarp();
  } else if (warp >= kSoftmaxWarp0 && warp < kSoftmaxWarpEnd) {
    sas::setmaxnreg_inc<kRegsSoftmax>();
    // =============================== softmax groups A (warps 4-7, heads 0-31)
    // and B (warps 8-11, heads 32-63) / epilogue
    const int quad = warp & 3;  // TMEM lane quadrant of this warp
    const int half = warp >= kSoftmaxWarpB ? 1 : 0;
    SmGroup G{32 * half, half, quad, lane, quad * 32 + lane, quad == 0,
              GroupSync{&bars[half ? B_LSYNC : B_SSYNC], reinterpret_cast<uint32_t*>(misc + (half ? M_LWORD : M_SWORD)),
                        0},
              {}, tmem + ((uint32_t)(quad * 32) << 16), 0};
    TileIter it;
    it.init(usp, *reinterpret_cast<const RangeInfo*>(misc + M_RANGE));
    Tile tl;
    Seg pend{};         // a complete token whose output rows are still to be written
    bool pending = false;
    uint32_t gtile = 0, gp = 0;
    bool ok = true;
    const bool trace_me = tracing && half == 0;
    unsigned long long trb[TR_NSLOTS];
    unsigned long long* trp = half == 0 ? tr : trb;
    while (ok && it.next(tl, tokp, p.n_win_chunks, p.scenario, p.ratio, p.K)) {
      for (int i = 0; ok && i < tl.nch; ++i)  // the tile's validity masks
        ok = twait(&bars[B_CFULL + (tl.g0 + i) % CD], ((tl.g0 + i) / CD) & 1, abort_flag, p.status, 8, trace_me,
                   trp[TR_S_WAIT_MASK]);
      float al;
      int need;
      if (ok)
        ok = tile_max_pass<DT>(p, G, sm, bars, cmask, gtile, tl.g0, tl.nch, tl.first, g, al, need, abort_flag,
                               trace_me, trp);
      if (TRACE && tid == kSoftmaxWarp0 * 32 && gtile < 2) ev(11 + gtile);
      for (int i = 0; ok && i < tl.nch; ++i) {
        ok = chunk_exp_pass<DT>(p, G, sm, bars, cmask, tl.g0 + i, i, i == 0 && need, tl.first, al, gp, abort_flag,
                                trace_me, trp);
        __syncwarp();
        if (lane == 0) sas::mbar_arrive(&bars[B_CEMPTY + (tl.g0 + i) % CD]);
        if (ok && i == 0 && pending) {
          ok = epilogue_second_half<DT, GA>(p, G, sm, bars, pend, g, abort_flag, trace_me, trp);
          pending = false;
        }
      }
      ++gtile;
      if (ok && tl.last) {
        if (it.sg.complete) {
          ok = epilogue_first_half<DT, GA>(p, G, sm, it.sg, g, abort_flag);
          pend = it.sg;
          pending = true;
        } else {
          ok = segment_epilogue<DT, GA>(p, G, sm, bars, it.sg, r, g, abort_flag, trace_me, trp);
        }
      }
    }
    if (TRACE && tid == kSoftmaxWarp0 * 32) ev(13);
    if (ok && pending) ok = epilogue_second_half<DT, GA>(p, G, sm, bars, pend, g, abort_flag, trace_me, trp);
    if (TRACE && tid == kSoftmaxWarp0 * 32) ev(14);
    if (FUSED && ok)
      zero_uncovered<DT, GA>(p, G, usp, tokp, reinterpret_cast<const int*>(smem + OFF_PLAN + P_SMAX),
                         *reinterpret_cast<const RangeInfo*>(misc + M_RANGE), g, abort_flag);
  } else {
    sas::setmaxnreg_dec<kRegsLean>();  // warps 14-15: idle
  }

  if (TRACE) {
    unsigned long long* tp = p.trace + (size_t)blockIdx.x * TR_NSLOTS;
    if (tid == kLoaderLeadWarp * 32) {
      tp[TR_P_WAIT_EMPTY] = tr[TR_P_WAIT_EMPTY];
      tp[TR_P_WAIT_MASK] = tr[TR_P_WAIT_MASK];
    } else if (tid == kCoordWarp * 32) {
      tp[TR_P_COORD] = tr[TR_P_COORD];
      tp[TR_P_ISSUE] = tr[TR_P_WAIT_MASK];  // the coordinate warp's wait for a free ring slot
    } else if (warp == kMmaWarp && lane == 0) {
      tp[TR_M_WAIT_Q] = tr[TR_M_WAIT_Q];
      tp[TR_M_WAIT_FULL] = tr[TR_M_WAIT_FULL];
      tp[TR_M_WAIT_P] = tr[TR_M_WAIT_P];
      tp[TR_M_WAIT_O] = tr[TR_M_WAIT_O];
      tp[TR_E_COPY] = tr[TR_E_COPY];
      tp[TR_S_SYNC1] = tr[TR_S_SYNC1];  // MMA: async-proxy fences
      tp[TR_S_SYNC2] = tr[TR_S_SYNC2];  // MMA: QK^T issue
      tp[TR_S_EXP] = tr[TR_S_EXP];      // MMA: P.V issue
    } else if (tid == kSoftmaxWarp0 * 32) {
      tp[TR_S_WAIT_MASK] = tr[TR_S_WAIT_MASK];
      tp[TR_S_WAIT_S] = tr[TR_S_WAIT_S];
      tp[TR_S_SOFTMAX] = tr[TR_S_SOFTMAX];
      tp[TR_S_WAIT_O] = tr[TR_S_WAIT_O];
      tp[TR_S_EPI] = tr[TR_S_EPI];
      tp[TR_CHUNKS] = tr[TR_CHUNKS];
      tp[TR_SEGS] = tr[TR_SEGS];
      tp[TR_TOTAL] = clock64() - t_start;
      tp[TR_FIRST_S] = tr[TR_FIRST_S] ? tr[TR_FIRST_S] - t_start : 0;
      tp[TR_PROLOGUE] = t_start - t_entry;
      tp[TR_E_TMEM] = tr[TR_E_TMEM];
      tp[TR_E_STAGE] = tr[TR_E_STAGE];
      tp[TR_E_RED] = tr[TR_E_RED];
      for (int i = TR_S_LD; i < TR_FIRST_S; ++i)
        if (i != TR_S_SYNC1 && i != TR_S_SYNC2 && i != TR_S_EXP) tp[i] = tr[i];
    }
  }
  sas::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    sas::tc_fence_after();
    sas::tmem_dealloc(tmem, TMEM_COLS);
  }
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

// Launch with programmatic stream serialization, so the kernel's prologue can
// overlap the previous kernel on the stream (the kernel calls pdl_wait()
// before reading what that kernel wrote).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Tuning / diagnostics knobs set through sas_fwd_set_option (process-wide).
float g_tau = 0.0f;  // exact running max (golden.py); > 0 only for experiments
int g_cut_cost = -1; // tokens are never split across CTAs unless set
unsigned long long* g_trace = nullptr;
size_t g_trace_bytes = 0;  // size of the trace buffer
int g_trace_dev = -1;      // the device that owns it
unsigned long long g_wait_ns = SAS_WAIT_LIMIT_NS;

struct WsLayout {
  size_t tok, unit, po, pl, cnt, od, total;
};
WsLayout ws_layout(int T, int H, int num_sms) {
  const int G = (H + HG - 1) / HG;
  const int R = std::max(1, num_sms / G);
  WsLayout w;
  w.tok = 0;
  w.unit = align_up(w.tok + sizeof(TokInfo) * (size_t)std::max(T, 1), 256);
  w.po = align_up(w.unit + sizeof(int32_t) * ((size_t)T + 1), 256);
  w.pl = align_up(w.po + sizeof(float) * (size_t)R * 2 * G * HG * D, 256);
  w.cnt = align_up(w.pl + sizeof(float) * (size_t)R * 2 * G * HG, 256);
  w.od = align_up(w.cnt + sizeof(int32_t) * (size_t)R * G * 2, 256);
  w.total = align_up(w.od + sizeof(OutDesc), 256);
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
      // value = the buffer's size in bytes; a launch on another device, or
      // whose grid needs more than that, is refused
      if (ptr == nullptr) {
        g_trace = nullptr;
        g_trace_bytes = 0;
        g_trace_dev = -1;
        return SAS_OK;
      }
      {
        cudaPointerAttributes a;
        if (!(value > 0.0) || cudaPointerGetAttributes(&a, ptr) != cudaSuccess || a.type != cudaMemoryTypeDevice) {
          cudaGetLastError();
          return SAS_ERR_INVALID_ARG;
        }
        g_trace = static_cast<unsigned long long*>(ptr);
        g_trace_bytes = (size_t)value;
        g_trace_dev = a.device;
      }
      return SAS_OK;
    case SAS_OPT_WAIT_LIMIT_NS:
      if (!(value >= 0.0 && value <= 60e9)) return SAS_ERR_INVALID_ARG;
      g_wait_ns = value == 0.0 ? SAS_WAIT_LIMIT_NS : (unsigned long long)value;
      return SAS_OK;
    case SAS_OPT_SCHED_SCAN_CAP:
      if (!(value >= 0.0 && value <= 4e18)) return SAS_ERR_INVALID_ARG;
      sas::set_sched_scan_cap((long long)value);
      return SAS_OK;
    case SAS_OPT_SPLIT_TOKENS:
      if (!(value >= -1.0 && value <= 1e6)) return SAS_ERR_INVALID_ARG;
      g_cut_cost = value < 0.0 ? -1 : (int)value;
      return SAS_OK;
    default:
      return SAS_ERR_INVALID_ARG;
  }
}

extern "C" size_t sas_fwd_workspace_bytes(int32_t num_tokens, int32_t num_heads, int32_t num_sms) {
  return ws_layout(num_tokens, num_heads, num_sms).total;
}

namespace {
// The forward; host_od != nullptr selects the head-sharded outputs (GA kernels).
int fwd_impl(const void* q, int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t dtype, int32_t layout_q,
             int32_t batch, int32_t max_seqlen_q, const int32_t* cu_seqlens_q, const int32_t* seqused_kv,
             const void* ori_kv, int64_t ori_num_blocks, int32_t ori_block_size, const int32_t* ori_block_table,
             int32_t ori_table_stride, const void* cmp_kv, int64_t cmp_num_blocks, int32_t cmp_block_size,
             const int32_t* cmp_block_table, int32_t cmp_table_stride, const int32_t* cmp_sparse_indices,
             int32_t topk, const float* sinks, const int32_t* metadata, float softmax_scale, int32_t cmp_ratio,
             int32_t ori_win_left, int32_t scenario, void* out, float* lse, const OutDesc* host_od, int32_t num_sms,
             int32_t stage_mask, int32_t* status, void* workspace, size_t workspace_bytes, void* stream) {
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
  // fused plan for small token counts (decode); early start only when the
  // caller guarantees the kernel before is sas_metadata of this call (the
  // CTA that shares an SM with the scheduler starts when it ends; measured,
  // that beats leaving the SM out of the grid)
  const bool fused = num_tokens <= kFusedMaxT;
  const bool early = fused && (stage_mask & SAS_FLAG_AFTER_METADATA);
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
  pp.merge_cnt = reinterpret_cast<int32_t*>(ws + wl.cnt);
  pp.n_cnt = R * G * 2;

  const OutDesc* god = nullptr;
  if (host_od) {
    // the output descriptor goes to the workspace, where the GA kernels read it
    god = reinterpret_cast<const OutDesc*>(ws + wl.od);
    if (cudaMemcpyAsync(ws + wl.od, host_od, sizeof(OutDesc), cudaMemcpyHostToDevice, st) != cudaSuccess)
      return SAS_ERR_CUDA;
  }
  pp.god = god;
  if ((stage_mask & SAS_STAGE_PLAN) && !fused) {
    if (launch_pdl(sas_plan_kernel, dim3(1), dim3(1024), 0, st, pp) != cudaSuccess) return SAS_ERR_CUDA;
  }
  if (!(stage_mask & SAS_STAGE_ATTENTION)) return SAS_OK;

  const CUtensorMapDataType tdt = dtype == SAS_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  alignas(64) CUtensorMap tm_q;
  const int q_box_h = std::min(HG, num_heads);
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
  fp.ori_nblk = (int)ori_num_blocks;
  fp.cmp_nblk = (int)(scenario >= 2 ? cmp_num_blocks : ori_num_blocks);
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
  fp.merge_cnt = pp.merge_cnt;

  fp.status = status;
  fp.q_box_h = q_box_h;
  fp.tau = g_tau;
  fp.cut_cost = g_cut_cost;
  fp.wait_ns = g_wait_ns;
  fp.fused = fused ? 1 : 0;
  fp.early = early ? 1 : 0;
  fp.B = batch;
  fp.S = max_seqlen_q;
  fp.layout = layout_q;
  fp.cu = cu_seqlens_q;
  fp.seqused_kv = seqused_kv;
  fp.meta = metadata;
  fp.trace = g_trace;
  fp.god = god;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SAS_ERR_CUDA;
  static uint64_t attr_done = 0;  // bit per device
  if (!(attr_done & (1ull << dev))) {
    const int a = cudaFuncAttributeMaxDynamicSharedMemorySize;
    if (cudaFuncSetAttribute(sas_fwd_kernel<0, false, false, false>, (cudaFuncAttribute)a, SMEM_BYTES_BASE) !=
            cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<1, false, false, false>, (cudaFuncAttribute)a, SMEM_BYTES_BASE) !=
            cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<0, true, false, false>, (cudaFuncAttribute)a, SMEM_BYTES_BASE) !=
            cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<1, true, false, false>, (cudaFuncAttribute)a, SMEM_BYTES_BASE) !=
            cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<0, false, true, false>, (cudaFuncAttribute)a, SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<1, false, true, false>, (cudaFuncAttribute)a, SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<0, true, true, false>, (cudaFuncAttribute)a, SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<1, true, true, false>, (cudaFuncAttribute)a, SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<0, false, false, true>, (cudaFuncAttribute)a, SMEM_BYTES_BASE) !=
            cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<1, false, false, true>, (cudaFuncAttribute)a, SMEM_BYTES_BASE) !=
            cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<0, false, true, true>, (cudaFuncAttribute)a, SMEM_BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(sas_fwd_kernel<1, false, true, true>, (cudaFuncAttribute)a, SMEM_BYTES) != cudaSuccess)
      return SAS_ERR_CUDA;
    attr_done |= 1ull << dev;
  }
  if (fp.trace && (dev != g_trace_dev || g_trace_bytes < (size_t)R * G * (TR_NSLOTS + 16) * sizeof(uint64_t)))
    return SAS_ERR_INVALID_ARG;
  if (stage_mask & SAS_STAGE_ATTENTION) {
    const bool tr = fp.trace != nullptr;
    const dim3 grid(R * G), block(kThreads);
    using KernelFn = void (*)(const CUtensorMap, const FwdParams);
    // [dtype][trace][fused]; head-sharded outputs: [dtype][fused] (no trace)
    static const KernelFn kernels[2][2][2] = {
        {{sas_fwd_kernel<0, false, false, false>, sas_fwd_kernel<0, false, true, false>},
         {sas_fwd_kernel<0, true, false, false>, sas_fwd_kernel<0, true, true, false>}},
        {{sas_fwd_kernel<1, false, false, false>, sas_fwd_kernel<1, false, true, false>},
         {sas_fwd_kernel<1, true, false, false>, sas_fwd_kernel<1, true, true, false>}}};
    static const KernelFn ga_kernels[2][2] = {
        {sas_fwd_kernel<0, false, false, true>, sas_fwd_kernel<0, false, true, true>},
        {sas_fwd_kernel<1, false, false, true>, sas_fwd_kernel<1, false, true, true>}};
    const int di = dtype == SAS_DTYPE_BF16 ? 0 : 1;
    const KernelFn k = god ? ga_kernels[di][fused ? 1 : 0] : kernels[di][tr ? 1 : 0][fused ? 1 : 0];
    const cudaError_t e = launch_pdl(k, grid, block, fused ? SMEM_BYTES : SMEM_BYTES_BASE, st, tm_q, fp);
    if (e != cudaSuccess) return SAS_ERR_CUDA;
  }
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}
}  // namespace

extern "C" int sas_sparse_attn_sharedkv_fwd(
    const void* q, int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t dtype, int32_t layout_q,
    int32_t batch, int32_t max_seqlen_q, const int32_t* cu_seqlens_q, const int32_t* seqused_kv, const void* ori_kv,
    int64_t ori_num_blocks, int32_t ori_block_size, const int32_t* ori_block_table, int32_t ori_table_stride,
    const void* cmp_kv, int64_t cmp_num_blocks, int32_t cmp_block_size, const int32_t* cmp_block_table,
    int32_t cmp_table_stride, const int32_t* cmp_sparse_indices, int32_t topk, const float* sinks,
    const int32_t* metadata, float softmax_scale, int32_t cmp_ratio, int32_t ori_win_left, int32_t scenario,
    void* out, float* lse, int32_t num_sms, int32_t stage_mask, int32_t* status, void* workspace,
    size_t workspace_bytes, void* stream) {
  return fwd_impl(q, num_tokens, num_heads, head_dim, dtype, layout_q, batch, max_seqlen_q, cu_seqlens_q, seqused_kv,
                  ori_kv, ori_num_blocks, ori_block_size, ori_block_table, ori_table_stride, cmp_kv, cmp_num_blocks,
                  cmp_block_size, cmp_block_table, cmp_table_stride, cmp_sparse_indices, topk, sinks, metadata,
                  softmax_scale, cmp_ratio, ori_win_left, scenario, out, lse, nullptr, num_sms, stage_mask, status,
                  workspace, workspace_bytes, stream);
}

extern "C" int sas_sparse_attn_sharedkv_fwd_gather(
    const void* q, int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t dtype, int32_t layout_q,
    int32_t batch, int32_t max_seqlen_q, const int32_t* cu_seqlens_q, const int32_t* seqused_kv, const void* ori_kv,
    int64_t ori_num_blocks, int32_t ori_block_size, const int32_t* ori_block_table, int32_t ori_table_stride,
    const void* cmp_kv, int64_t cmp_num_blocks, int32_t cmp_block_size, const int32_t* cmp_block_table,
    int32_t cmp_table_stride, const int32_t* cmp_sparse_indices, int32_t topk, const float* sinks,
    const int32_t* metadata, float softmax_scale, int32_t cmp_ratio, int32_t ori_win_left, int32_t scenario,
    void* const* outs, float* const* lses, int32_t n_out, int32_t out_heads_total, int32_t out_head_offset,
    int32_t num_sms, int32_t stage_mask, int32_t* status, void* workspace, size_t workspace_bytes, void* stream) {
  if (!outs || n_out < 1 || n_out > kMaxOut || out_head_offset < 0 || out_heads_total < out_head_offset + num_heads)
    return SAS_ERR_INVALID_ARG;
  if (stage_mask & SAS_FLAG_AFTER_METADATA) return SAS_ERR_INVALID_ARG;
  if (g_cut_cost >= 0 || g_trace) return SAS_ERR_UNSUPPORTED;  // split tokens merge through one output
  OutDesc od{};
  for (int k = 0; k < n_out; ++k) {
    if (!outs[k] || (lses && !lses[k])) return SAS_ERR_INVALID_ARG;
    od.out[k] = static_cast<uint8_t*>(outs[k]);
    od.lse[k] = lses ? lses[k] : nullptr;
  }
  od.n = n_out;
  od.H_total = out_heads_total;
  od.h0 = out_head_offset;
  return fwd_impl(q, num_tokens, num_heads, head_dim, dtype, layout_q, batch, max_seqlen_q, cu_seqlens_q, seqused_kv,
                  ori_kv, ori_num_blocks, ori_block_size, ori_block_table, ori_table_stride, cmp_kv, cmp_num_blocks,
                  cmp_block_size, cmp_block_table, cmp_table_stride, cmp_sparse_indices, topk, sinks, metadata,
                  softmax_scale, cmp_ratio, ori_win_left, scenario, outs[0], lses ? lses[0] : nullptr, &od, num_sms,
                  stage_mask, status, workspace, workspace_bytes, stream);
}
