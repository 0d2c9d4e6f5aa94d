// Backward of the sparse shared-KV attention (sm_100a), consuming the
// forward's log-sum-exp.
//
// The reference documents the LSE output as the input of a FlashAttention-2
// style backward (sparse_attn_sharedkv_tilelang/api.py:32-35, 176-184) but
// ships none. This is that backward for the forward's semantics
// (golden.py:69-204): per query token t and head h the attended rows are the
// window [max(s_g - win_left, 0), s_g] of the raw cache, then the compressed
// rows (the first min(K, threshold) top-k slots, stopping at the first -1,
// skipping ids outside [0, threshold); all of [0, threshold) for the dense
// scenario), with K = V (one row serves as key and value) and a per-head
// sink logit in the softmax denominator. With s_j = scale * q.k_j,
// p_j = exp(s_j - lse), p_sink = exp(sink - lse) and D = sum_d dO * O:
//   dS_j   = p_j (dO.k_j - D)
//   dq     = scale * sum_j dS_j k_j
//   dkv_j += scale * dS_j q + p_j dO      (k_j is both key and value)
//   dsink -= p_sink D
// The gradient is that of the exact softmax (P is not rounded to the I/O
// type, unlike the forward's P.V, golden.py:191-195).
//
// One CTA per (token, group of 16 heads), 256 threads, fp32 math on the CUDA
// cores, the token's rows walked in chunks of 32. dq is written once per
// token; the row gradients are accumulated with fp32 vector atomics into
// caller-provided fp32 buffers shaped like the pools (a row can be attended
// by many tokens and heads), and sas_bwd_cast converts them to the I/O type.
#include <algorithm>
#include <cstdint>

#include "sas_common.cuh"

namespace {

constexpr int D = 512;
constexpr int BH = 16;     // heads per CTA
constexpr int BR = 32;     // rows per chunk
constexpr int kThreads = 256;
constexpr int kSmemBytes = (2 * BH + BR) * D * 4;  // q, dO and the row chunk, fp32

struct BwdParams {
  int T, H, B, S, layout, scenario, K, ratio, win_left;
  int ori_bs, ori_bt_stride, cmp_bs, cmp_bt_stride, ori_nblk, cmp_nblk;
  const uint16_t* q;
  const uint16_t* out;
  const uint16_t* dout;
  const float* lse;
  const uint16_t* ori_kv;
  const uint16_t* cmp_kv;
  const int32_t* ori_bt;
  const int32_t* cmp_bt;
  const int32_t* idx;
  const int32_t* cu;
  const int32_t* seqused_kv;
  const float* sinks;
  float scale;
  uint16_t* dq;
  float* d_ori;   // [ori_nblk * ori_bs, 512]
  float* d_cmp;   // [cmp_nblk * cmp_bs, 512]
  float* dsinks;  // [H]
  int32_t* status;
};

template <int DT>
__device__ __forceinline__ float to_f(uint16_t v) {
  if constexpr (DT == 0) return __uint_as_float((uint32_t)v << 16);
  else return __half2float(__ushort_as_half(v));
}
template <int DT>
__device__ __forceinline__ uint16_t from_f(float x) {
  if constexpr (DT == 0) return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  else return __half_as_ushort(__float2half_rn(x));
}

__device__ __forceinline__ int py_floordiv(int a, int b) {
  int q = a / b, r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) --q;
  return q;
}

template <int DT>
__global__ void __launch_bounds__(kThreads, 1) sas_bwd_kernel(const BwdParams p) {
  extern __shared__ __align__(16) float smem_f[];
  float (*qs)[D] = reinterpret_cast<float (*)[D]>(smem_f);                  // [BH][D]
  float (*dos)[D] = reinterpret_cast<float (*)[D]>(smem_f + BH * D);        // [BH][D]
  float (*ks)[D] = reinterpret_cast<float (*)[D]>(smem_f + 2 * BH * D);     // [BR][D]
  __shared__ float Ps[BR][BH + 1];
  __shared__ float DSs[BR][BH + 1];
  __shared__ float lse_s[BH], D_s[BH];
  __shared__ int rows_s[BR];
  __shared__ int first_neg;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t = blockIdx.x, h0 = blockIdx.y * BH;
  const int nh = min(BH, p.H - h0);

  // token -> (request, position): the forward's layout rules (api.py:208-240)
  int b, s, act_q;
  if (p.layout == SAS_LAYOUT_TND) {
    int lo = 0, hi = p.B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.cu[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    b = lo;
    s = t - p.cu[b];
    act_q = p.cu[b + 1] - p.cu[b];
  } else {
    b = t / p.S;
    s = t - b * p.S;
    act_q = p.cu ? p.cu[b + 1] - p.cu[b] : p.S;
  }
  const bool live = b < p.B && s < act_q && s >= 0;
  const int s_g = live ? p.seqused_kv[b] - act_q + s : -1;
  const int thr = max(py_floordiv(s_g + 1, p.ratio), 0);

  // q, dO and O rows of this token's heads; D = sum_d dO * O per head
  for (int i = tid; i < BH * D; i += kThreads) {
    const int hh = i / D, d = i % D;
    float qv = 0.f, dv = 0.f;
    if (hh < nh && live) {
      const size_t o = ((size_t)t * p.H + h0 + hh) * D + d;
      qv = to_f<DT>(p.q[o]);
      dv = to_f<DT>(p.dout[o]);
    }
    qs[hh][d] = qv;
    dos[hh][d] = dv;
  }
  if (tid == 0) first_neg = INT32_MAX;
  __syncthreads();
  for (int hh = warp; hh < BH; hh += kThreads / 32) {
    float acc = 0.f;
    if (hh < nh && live) {
      const uint16_t* op = p.out + ((size_t)t * p.H + h0 + hh) * D;
      for (int d = lane; d < D; d += 32) acc += dos[hh][d] * to_f<DT>(op[d]);
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      D_s[hh] = acc;
      lse_s[hh] = (hh < nh && live) ? p.lse[(size_t)t * p.H + h0 + hh] : 0.f;
    }
  }
  // compressed scan limit: the first -1 among the first min(K, thr) slots
  // (golden.py:55-56)
  const int n_slots = p.scenario == 3 ? min(p.K, thr) : (p.scenario == 2 ? thr : 0);
  if (p.scenario == 3 && live)
    for (int i = tid; i < n_slots; i += kThreads)
      if (p.idx[(size_t)t * p.K + i] == -1) atomicMin(&first_neg, i);
  __syncthreads();
  if (live && tid < nh) {
    const int h = h0 + tid;
    const float ps = __expf(p.sinks[h] - lse_s[tid]);
    atomicAdd(&p.dsinks[h], -ps * D_s[tid]);
  }

  const int win_lo = max(s_g - p.win_left, 0);
  const int n_win = (live && s_g >= 0) ? s_g - win_lo + 1 : 0;
  const int n_cmp = live ? (p.scenario == 3 ? min(n_slots, first_neg) : n_slots) : 0;
  const int n_win_chunks = (n_win + BR - 1) / BR;
  const int n_chunks = n_win_chunks + (n_cmp + BR - 1) / BR;

  // this thread's share of dq: head dh, columns [dc * 32, dc * 32 + 32)
  const int dh = tid >> 4, dc = tid & 15;
  float dq[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) dq[i] = 0.f;
  bool bad = false;

  for (int c = 0; c < n_chunks; ++c) {
    const bool is_win = c < n_win_chunks;
    if (tid < BR) {
      int row = -1;
      if (is_win) {
        const int j = c * BR + tid;
        if (j < n_win) {
          const int pos = win_lo + j;
          const int col = pos / p.ori_bs;
          const int blk = col < p.ori_bt_stride ? p.ori_bt[(size_t)b * p.ori_bt_stride + col] : -1;
          bad |= col >= p.ori_bt_stride || blk >= p.ori_nblk;
          if (blk >= 0 && blk < p.ori_nblk) row = blk * p.ori_bs + pos % p.ori_bs;
        }
      } else {
        const int j = (c - n_win_chunks) * BR + tid;
        if (j < n_cmp) {
          const int id = p.scenario == 3 ? p.idx[(size_t)t * p.K + j] : j;
          if (id >= 0 && id < thr) {
            const int col = id / p.cmp_bs;
            const int blk = col < p.cmp_bt_stride ? p.cmp_bt[(size_t)b * p.cmp_bt_stride + col] : -1;
            bad |= col >= p.cmp_bt_stride || blk >= p.cmp_nblk;
            if (blk >= 0 && blk < p.cmp_nblk) row = blk * p.cmp_bs + id % p.cmp_bs;
          }
        }
      }
      rows_s[tid] = row;
    }
    __syncthreads();
    const uint16_t* pool = is_win ? p.ori_kv : p.cmp_kv;
    for (int i = tid; i < BR * D / 8; i += kThreads) {
      const int j = i / (D / 8), d8 = (i % (D / 8)) * 8;
      const int row = rows_s[j];
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (row >= 0) {
        const uint4 raw = *reinterpret_cast<const uint4*>(pool + (size_t)row * D + d8);
        const uint16_t* e = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = to_f<DT>(e[k]);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) ks[j][d8 + k] = v[k];
    }
    __syncthreads();
    // scores and dP: thread -> row j = tid / 8, heads hp and hp + 8
    {
      const int j = tid >> 3, hp = tid & 7;
      float s0 = 0.f, s1 = 0.f, g0 = 0.f, g1 = 0.f;
#pragma unroll 4
      for (int d = 0; d < D; ++d) {
        const float kv = ks[j][d];
        s0 += qs[hp][d] * kv;
        s1 += qs[hp + 8][d] * kv;
        g0 += dos[hp][d] * kv;
        g1 += dos[hp + 8][d] * kv;
      }
      const bool v = rows_s[j] >= 0;
      const float p0 = v && hp < nh ? __expf(s0 * p.scale - lse_s[hp]) : 0.f;
      const float p1 = v && hp + 8 < nh ? __expf(s1 * p.scale - lse_s[hp + 8]) : 0.f;
      Ps[j][hp] = p0;
      Ps[j][hp + 8] = p1;
      DSs[j][hp] = p0 * (g0 - D_s[hp]);
      DSs[j][hp + 8] = p1 * (g1 - D_s[hp + 8]);
    }
    __syncthreads();
    // dq += dS . K for head dh, 32 columns
#pragma unroll 4
    for (int j = 0; j < BR; ++j) {
      const float ds = DSs[j][dh];
#pragma unroll
      for (int i = 0; i < 32; ++i) dq[i] += ds * ks[j][dc * 32 + i];
    }
    // dkv_j = scale * dS_j . Q + P_j . dO: thread -> row j = tid / 8, 64 columns
    {
      const int j = tid >> 3, c0 = (tid & 7) * 64;
      const int row = rows_s[j];
      if (row >= 0) {
        float* dst = (is_win ? p.d_ori : p.d_cmp) + (size_t)row * D + c0;
#pragma unroll 1
        for (int q4 = 0; q4 < 16; ++q4) {
          float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
          for (int hh = 0; hh < BH; ++hh) {
            const float ds = DSs[j][hh] * p.scale, pp = Ps[j][hh];
            const int d = c0 + q4 * 4;
            a.x += ds * qs[hh][d] + pp * dos[hh][d];
            a.y += ds * qs[hh][d + 1] + pp * dos[hh][d + 1];
            a.z += ds * qs[hh][d + 2] + pp * dos[hh][d + 2];
            a.w += ds * qs[hh][d + 3] + pp * dos[hh][d + 3];
          }
          atomicAdd(reinterpret_cast<float4*>(dst + q4 * 4), a);
        }
      }
    }
    __syncthreads();
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0 && p.status) atomicCAS(p.status, 0, SAS_ERR_BAD_BLOCK_ENTRY);
  if (dh < nh) {
    uint16_t* o = p.dq + ((size_t)t * p.H + h0 + dh) * D + dc * 32;
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = from_f<DT>(dq[i] * p.scale);
  }
}

template <int DT>
__global__ void sas_bwd_cast_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = from_f<DT>(src[i]);
}

}  // namespace

extern "C" int sas_sparse_attn_sharedkv_bwd(
    const void* dout, const void* q, const void* out, const float* lse, int32_t num_tokens, int32_t num_heads,
    int32_t head_dim, int32_t dtype, int32_t layout_q, int32_t batch, int32_t max_seqlen_q,
    const int32_t* cu_seqlens_q, const int32_t* seqused_kv, const void* ori_kv, int64_t ori_num_blocks,
    int32_t ori_block_size, const int32_t* ori_block_table, int32_t ori_table_stride, const void* cmp_kv,
    int64_t cmp_num_blocks, int32_t cmp_block_size, const int32_t* cmp_block_table, int32_t cmp_table_stride,
    const int32_t* cmp_sparse_indices, int32_t topk, const float* sinks, float softmax_scale, int32_t cmp_ratio,
    int32_t ori_win_left, int32_t scenario, void* dq, float* d_ori_kv, float* d_cmp_kv, float* d_sinks,
    int32_t* status, void* stream) {
  if (head_dim != D) return SAS_ERR_UNSUPPORTED;
  if (num_heads <= 0) return SAS_ERR_UNSUPPORTED;
  if (dtype != SAS_DTYPE_BF16 && dtype != SAS_DTYPE_FP16) return SAS_ERR_UNSUPPORTED;
  if (scenario < 1 || scenario > 3) return SAS_ERR_INVALID_ARG;
  if (num_tokens < 0 || batch < 0 || !dout || !q || !out || !lse || !seqused_kv || !ori_kv || !ori_block_table ||
      !sinks || !dq || !d_ori_kv || !d_sinks)
    return SAS_ERR_INVALID_ARG;
  if (layout_q == SAS_LAYOUT_TND && !cu_seqlens_q) return SAS_ERR_INVALID_ARG;
  if (layout_q == SAS_LAYOUT_BSND && (int64_t)batch * max_seqlen_q != num_tokens) return SAS_ERR_INVALID_ARG;
  if (layout_q != SAS_LAYOUT_TND && layout_q != SAS_LAYOUT_BSND) return SAS_ERR_UNSUPPORTED;
  if (ori_win_left < 0) return SAS_ERR_UNSUPPORTED;
  if (scenario >= 2 && (!cmp_kv || !cmp_block_table || !d_cmp_kv || cmp_ratio <= 0 || cmp_block_size <= 0))
    return SAS_ERR_INVALID_ARG;
  if (scenario == 3 && (!cmp_sparse_indices || topk <= 0)) return SAS_ERR_INVALID_ARG;
  if (ori_block_size <= 0) return SAS_ERR_INVALID_ARG;
  if ((int64_t)ori_num_blocks * ori_block_size >= (1LL << 31) ||
      (scenario >= 2 && (int64_t)cmp_num_blocks * cmp_block_size >= (1LL << 31)))
    return SAS_ERR_UNSUPPORTED;
  if (!sas::select_device_of(q)) return SAS_ERR_INVALID_ARG;
  if (num_tokens == 0 || batch == 0) return SAS_OK;
  BwdParams p{};
  p.T = num_tokens;
  p.H = num_heads;
  p.B = batch;
  p.S = max_seqlen_q;
  p.layout = layout_q;
  p.scenario = scenario;
  p.K = scenario == 3 ? topk : 0;
  p.ratio = scenario >= 2 ? cmp_ratio : 1;
  p.win_left = ori_win_left;
  p.ori_bs = ori_block_size;
  p.ori_bt_stride = ori_table_stride;
  p.cmp_bs = scenario >= 2 ? cmp_block_size : 1;
  p.cmp_bt_stride = cmp_table_stride;
  p.ori_nblk = (int)ori_num_blocks;
  p.cmp_nblk = scenario >= 2 ? (int)cmp_num_blocks : 0;
  p.q = static_cast<const uint16_t*>(q);
  p.out = static_cast<const uint16_t*>(out);
  p.dout = static_cast<const uint16_t*>(dout);
  p.lse = lse;
  p.ori_kv = static_cast<const uint16_t*>(ori_kv);
  p.cmp_kv = static_cast<const uint16_t*>(scenario >= 2 ? cmp_kv : ori_kv);
  p.ori_bt = ori_block_table;
  p.cmp_bt = cmp_block_table;
  p.idx = cmp_sparse_indices;
  p.cu = cu_seqlens_q;
  p.seqused_kv = seqused_kv;
  p.sinks = sinks;
  p.scale = softmax_scale;
  p.dq = static_cast<uint16_t*>(dq);
  p.d_ori = d_ori_kv;
  p.d_cmp = d_cmp_kv;
  p.dsinks = d_sinks;
  p.status = status;
  const dim3 grid(num_tokens, (num_heads + BH - 1) / BH);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto a = cudaFuncAttributeMaxDynamicSharedMemorySize;
  if (cudaFuncSetAttribute(sas_bwd_kernel<0>, a, kSmemBytes) != cudaSuccess ||
      cudaFuncSetAttribute(sas_bwd_kernel<1>, a, kSmemBytes) != cudaSuccess)
    return SAS_ERR_CUDA;
  if (dtype == SAS_DTYPE_BF16) sas_bwd_kernel<0><<<grid, kThreads, kSmemBytes, st>>>(p);
  else sas_bwd_kernel<1><<<grid, kThreads, kSmemBytes, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}

extern "C" int sas_bwd_cast(const float* src, void* dst, int64_t n, int32_t dtype, void* stream) {
  if (!src || !dst || n < 0) return SAS_ERR_INVALID_ARG;
  if (dtype != SAS_DTYPE_BF16 && dtype != SAS_DTYPE_FP16) return SAS_ERR_UNSUPPORTED;
  if (n == 0) return SAS_OK;
  if (!sas::select_device_of(src)) return SAS_ERR_INVALID_ARG;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == SAS_DTYPE_BF16)
    sas_bwd_cast_kernel<0><<<blocks, 256, 0, st>>>(src, static_cast<uint16_t*>(dst), (size_t)n);
  else
    sas_bwd_cast_kernel<1><<<blocks, 256, 0, st>>>(src, static_cast<uint16_t*>(dst), (size_t)n);
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}
