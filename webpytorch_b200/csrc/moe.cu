// Mixture-of-experts block on B200: device-side routing and the element-wise glue around the
// grouped expert GEMMs.
//
// Reference semantics (webtorch/lm_engine.py:294-333, moe_mlp): probabilities = softmax over
// all experts of the router logits (float64 on the host there); the top_k experts of each token
// are selected (argpartition), their probabilities optionally renormalised to sum to one, every
// expert runs down(silu(gate(x)) * up(x)) over its tokens, and each token's output is the
// weighted sum of its experts' outputs.
//
// Here everything is on the device, so a decode step needs no host round trip and can be
// captured in a CUDA graph:
//   1. moe_topk_kernel      one warp per token: softmax statistics, top-k by repeated warp
//                           argmax (ties to the lower expert index), weights, per-expert counts
//   2. moe_scan_kernel      exclusive scan of the counts -> expert row offsets, the list of
//                           active experts, and the tile table of the grouped tensor-core GEMM
//   3. moe_scatter_kernel   each (token, k) pair takes a row of its expert's segment
//   4. grouped GEMMs over the permuted rows (gptq_gemv_tma.cu / gptq_gemm_sm100.cu)
//   5. moe_act_kernel       a = silu(gate) * up on the fused gate|up output
//   6. moe_combine_kernel   out[t] = sum_j w[t, j] * y[row(t, j)], in a fixed j order
// Rows inside an expert's segment are assigned with atomics, so their order varies from run to
// run, but no output value depends on it: every row is computed independently and the combine
// sums each token's k rows in slot order.
#include "ql_common.cuh"

namespace ql {
namespace {

constexpr int kMaxTopK = 16;
constexpr int kMaxExperts = 1024;

// Top-k of one token's logits by one warp: softmax statistics over all E experts in float64,
// then k rounds of warp argmax (ties to the lower expert index). Lane j < k returns pick j in
// (*idx, *w); the weights are the softmax probabilities, renormalised over the k when norm.
//
// Up to 32 * VPL experts every lane keeps its VPL logits and their exp(l - max) in registers: a
// pick is struck from its lane's bitmask and its probability comes from the lane that holds it,
// so a token costs VPL float64 exponentials per lane. Same arithmetic and order as the generic
// form below (identical results).
template <int VPL>
__device__ __forceinline__ void topk_token_reg(const float* __restrict__ row, int E, int k, int norm, int lane,
                                               int* idx, float* w) {
  float v[VPL];
  double ex[VPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? row[e] : -INFINITY;
    if (e < E) mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  double den = 0.0;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    ex[i] = lane + 32 * i < E ? exp((double)v[i] - (double)mx) : 0.0;
    den += ex[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  unsigned taken = 0u;
  double psum = 0.0, mine = 0.0;
  int my_idx = 0;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    double be = 0.0;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((taken >> i) & 1u) && (v[i] > best || (v[i] == best && e < bi))) {
        best = v[i];
        bi = e;
        be = ex[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const double oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
        be = oe;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    const double p = be / den;
    psum += p;
    if (lane == j) {
      my_idx = bi;
      mine = p;
    }
  }
  *idx = lane < k ? my_idx : 0;
  *w = lane < k ? (float)(norm ? mine / psum : mine) : 0.f;
}

// Any E (up to kMaxExperts): the logits are re-read from memory each round.
__device__ __forceinline__ void topk_token_any(const float* __restrict__ row, int E, int k, int norm, int lane,
                                               int* idx, float* w) {
  float mx = -INFINITY;
  for (int e = lane; e < E; e += 32) mx = fmaxf(mx, row[e]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  double den = 0.0;
  for (int e = lane; e < E; e += 32) den += exp((double)row[e] - (double)mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  int chosen[kMaxTopK];
  double psum = 0.0, mine = 0.0;
  int my_idx = 0;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      bool taken = false;
      for (int q = 0; q < j; ++q) taken |= (chosen[q] == e);
      const float v = row[e];
      if (!taken && (v > best || (v == best && e < bi))) {
        best = v;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    chosen[j] = bi;
    const double p = exp((double)best - (double)mx) / den;
    psum += p;
    if (lane == j) {
      my_idx = bi;
      mine = p;
    }
  }
  *idx = lane < k ? my_idx : 0;
  *w = lane < k ? (float)(norm ? mine / psum : mine) : 0.f;
}

__device__ __forceinline__ void topk_token(const float* __restrict__ row, int E, int k, int norm, int lane, int* idx,
                                           float* w) {
  if (E <= 128) topk_token_reg<4>(row, E, k, norm, lane, idx, w);
  else if (E <= 256) topk_token_reg<8>(row, E, k, norm, lane, idx, w);
  else topk_token_any(row, E, k, norm, lane, idx, w);
}

__global__ void moe_topk_kernel(const float* __restrict__ logits, int T, int E, int k, int norm,
                                int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
                                int32_t* __restrict__ counts) {
  const int warps = blockDim.x >> 5;
  const int t = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  int my;
  float w;
  topk_token(logits + (long)t * E, E, k, norm, lane, &my, &w);
  if (lane < k) {
    topk_idx[(long)t * k + lane] = my;
    topk_w[(long)t * k + lane] = w;
    atomicAdd(&counts[my], 1);
  }
}

// Block-wide scans over one thread per expert (blockDim >= E, a multiple of 32): exclusive
// scans of the row counts (-> segment offsets), of the active flags (-> compact active-expert
// list) and of the tile counts (-> the grouped matmul's tile table of `tile_rows`-row tiles).
// Every thread of the block calls it; thread e gets its expert's offset back.
__device__ int scan_experts(int c, int E, int tile_rows, int32_t* __restrict__ offsets, int32_t* __restrict__ active,
                            int32_t* __restrict__ n_active, int32_t* __restrict__ tiles, int32_t* __restrict__ n_tiles,
                            int max_tiles) {
  __shared__ int s_tot[3][32];
  const int e = threadIdx.x, lane = e & 31, w = e >> 5, nw = (blockDim.x + 31) >> 5;
  const int v[3] = {c, c > 0 ? 1 : 0, (c + tile_rows - 1) / tile_rows};
  int inc[3] = {v[0], v[1], v[2]};
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const int t = __shfl_up_sync(0xffffffffu, inc[q], o);
      if (lane >= o) inc[q] += t;
    }
  }
  if (lane == 31)
    for (int q = 0; q < 3; ++q) s_tot[q][w] = inc[q];
  __syncthreads();
  if (w == 0) {
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const int own = lane < nw ? s_tot[q][lane] : 0;
      int x = own;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
      }
      if (lane < nw) s_tot[q][lane] = x - own;   // exclusive warp base
    }
  }
  __syncthreads();
  int ex[3];
#pragma unroll
  for (int q = 0; q < 3; ++q) ex[q] = s_tot[q][w] + inc[q] - v[q];
  if (e < E) {
    offsets[e] = ex[0];
    if (c > 0) active[ex[1]] = e;
    for (int i = 0; i < v[2]; ++i) {
      const int ti = ex[2] + i;
      if (ti < max_tiles) {
        tiles[2 * ti] = e;
        tiles[2 * ti + 1] = i * tile_rows;
      }
    }
    if (e == E - 1) {
      offsets[E] = ex[0] + c;
      *n_active = ex[1] + v[1];
      const int nt = ex[2] + v[2];
      *n_tiles = nt < max_tiles ? nt : max_tiles;
    }
  }
  return ex[0];
}

__global__ void __launch_bounds__(1024) moe_scan_kernel(const int32_t* __restrict__ counts, int E, int tile_rows,
                                                        int32_t* __restrict__ offsets, int32_t* __restrict__ cursor,
                                                        int32_t* __restrict__ active, int32_t* __restrict__ n_active,
                                                        int32_t* __restrict__ tiles, int32_t* __restrict__ n_tiles,
                                                        int max_tiles) {
  const int e = threadIdx.x;
  const int c = e < E ? counts[e] : 0;
  scan_experts(c, E, tile_rows, offsets, active, n_active, tiles, n_tiles, max_tiles);
  if (e < E) cursor[e] = 0;
}

__global__ void moe_scatter_kernel(const int32_t* __restrict__ topk_idx, int T, int k, const int32_t* __restrict__ offsets,
                                   int32_t* __restrict__ cursor, int32_t* __restrict__ row_token,
                                   int32_t* __restrict__ pair_row) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * k) return;
  const int e = topk_idx[i];
  const int r = offsets[e] + atomicAdd(&cursor[e], 1);
  row_token[r] = i / k;
  pair_row[i] = r;
}

// The whole route in one CTA for decode-sized batches (T <= kSmallTokens, T * k <= kSmallPairs,
// E <= 1024): top-k per token (one warp each), histogram in shared memory, the scans, and the
// scatter.
constexpr int kSmallPairs = 4096;
// Above this many tokens the top-k runs on many SMs (one CTA holds the route of a decode step;
// a larger batch would queue all its tokens on one SM's warps).
constexpr int kSmallTokens = 64;
__global__ void __launch_bounds__(1024) moe_route_small_kernel(const float* __restrict__ logits, int T, int E, int k,
                                                               int norm, int tile_rows, int32_t* __restrict__ topk_idx,
                                                               float* __restrict__ topk_w, int32_t* __restrict__ counts,
                                                               int32_t* __restrict__ offsets, int32_t* __restrict__ active,
                                                               int32_t* __restrict__ n_active, int32_t* __restrict__ tiles,
                                                               int32_t* __restrict__ n_tiles, int max_tiles,
                                                               int32_t* __restrict__ row_token,
                                                               int32_t* __restrict__ pair_row) {
  __shared__ int s_cnt[1024];
  __shared__ int s_off[1024];
  __shared__ int s_idx[kSmallPairs];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  if (tid < E) s_cnt[tid] = 0;
  __syncthreads();
  for (int t = warp; t < T; t += nw) {
    int my;
    float w;
    topk_token(logits + (long)t * E, E, k, norm, lane, &my, &w);
    if (lane < k) {
      topk_idx[(long)t * k + lane] = my;
      topk_w[(long)t * k + lane] = w;
      s_idx[t * k + lane] = my;
      atomicAdd(&s_cnt[my], 1);
    }
  }
  __syncthreads();
  const int c = tid < E ? s_cnt[tid] : 0;
  if (tid < E) counts[tid] = c;
  const int off = scan_experts(c, E, tile_rows, offsets, active, n_active, tiles, n_tiles, max_tiles);
  if (tid < E) {
    s_off[tid] = off;
    s_cnt[tid] = 0;   // becomes the scatter cursor
  }
  __syncthreads();
  for (int i = tid; i < T * k; i += blockDim.x) {
    const int e = s_idx[i];
    const int r = s_off[e] + atomicAdd(&s_cnt[e], 1);
    row_token[r] = i / k;
    pair_row[i] = r;
  }
}

// Histogram of given group ids (expert-parallel dispatch and the receiving side's local grouping).
__global__ void moe_hist_kernel(const int32_t* __restrict__ ids, int n, int32_t* __restrict__ counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) atomicAdd(&counts[ids[i]], 1);
}

// a[r, n] = silu(y[r, n]) * y[r, I + n]  (gate | up fused along columns), silu = v * sigmoid(v)
__global__ void moe_act_kernel(const float* __restrict__ y, long P, int I, void* __restrict__ a, int a_dtype) {
  const long total = P * I;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long r = i / I;
    const int n = (int)(i - r * I);
    const float g = y[r * 2 * I + n];
    const float u = y[r * 2 * I + I + n];
    const float s = g / (1.0f + expf(-g));
    store_from_float(a, a_dtype, i, s * u);
  }
}

// out[t, h] = sum_j w[t, j] * z[pair_row[t, j], h]  (+ g[t] * shared[t, h], g = sigmoid of the
// shared-expert gate logit when given, else 1)
__global__ void moe_combine_kernel(const float* __restrict__ z, const int32_t* __restrict__ pair_row,
                                   const float* __restrict__ topk_w, int T, int k, int H,
                                   const float* __restrict__ shared, long lds, const float* __restrict__ shared_gate,
                                   long ldg, void* __restrict__ out, int out_dtype, long ldo) {
  const long total = (long)T * H;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int t = (int)(i / H);
    const int h = (int)(i - (long)t * H);
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc = fmaf(topk_w[(long)t * k + j], z[(long)pair_row[(long)t * k + j] * H + h], acc);
    if (shared) {
      float g = 1.f;
      if (shared_gate) g = 1.0f / (1.0f + expf(-shared_gate[(long)t * ldg]));
      acc += g * shared[(long)t * lds + h];
    }
    store_from_float(out, out_dtype, (long)t * ldo + h, acc);
  }
}

// The same sums (same order) four columns per thread, for H % 4 == 0 and 16-byte aligned rows:
// CTA b covers token b / parts, columns [(b % parts) * 1024, +1024); each thread's k row loads
// are independent 16-byte loads.
__global__ void __launch_bounds__(256) moe_combine4_kernel(const float* __restrict__ z,
                                                           const int32_t* __restrict__ pair_row,
                                                           const float* __restrict__ topk_w, int k, int H, int parts,
                                                           const float* __restrict__ shared, long lds,
                                                           const float* __restrict__ shared_gate, long ldg,
                                                           void* __restrict__ out, int out_dtype, long ldo) {
  const int t = blockIdx.x / parts;
  const int c4 = (blockIdx.x - t * parts) * blockDim.x + threadIdx.x;
  if (c4 * 4 >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int j = 0; j < k; ++j) {
    const float w = topk_w[(long)t * k + j];
    const float4 v = reinterpret_cast<const float4*>(z + (long)pair_row[(long)t * k + j] * H)[c4];
    acc.x = fmaf(w, v.x, acc.x);
    acc.y = fmaf(w, v.y, acc.y);
    acc.z = fmaf(w, v.z, acc.z);
    acc.w = fmaf(w, v.w, acc.w);
  }
  if (shared) {
    float g = 1.f;
    if (shared_gate) g = 1.0f / (1.0f + expf(-shared_gate[(long)t * ldg]));
    const float4 v = reinterpret_cast<const float4*>(shared + (long)t * lds)[c4];
    acc.x += g * v.x;
    acc.y += g * v.y;
    acc.z += g * v.z;
    acc.w += g * v.w;
  }
  const long o = (long)t * ldo + 4L * c4;
  if (out_dtype == QL_F32 && ((reinterpret_cast<uintptr_t>(out) | (uintptr_t)ldo * 4) & 15) == 0) {
    reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + o)[0] = acc;
  } else {
    store_from_float(out, out_dtype, o, acc.x);
    store_from_float(out, out_dtype, o + 1, acc.y);
    store_from_float(out, out_dtype, o + 2, acc.z);
    store_from_float(out, out_dtype, o + 3, acc.w);
  }
}

}  // namespace
}  // namespace ql

using namespace ql;

extern "C" int ql_moe_route(const float* logits, int T, int E, int top_k, int norm_topk_prob, int tile_rows,
                            int32_t* topk_idx, float* topk_w, int32_t* counts, int32_t* offsets, int32_t* cursor,
                            int32_t* active, int32_t* n_active, int32_t* tiles, int32_t* n_tiles, int max_tiles,
                            int32_t* row_token, int32_t* pair_row, void* stream) {
  if (T < 0 || E <= 0 || E > kMaxExperts || top_k <= 0 || top_k > E || top_k > kMaxTopK || tile_rows <= 0 ||
      max_tiles < 0) {
    set_error("ql_moe_route: bad sizes (T=%d E=%d top_k=%d; E <= %d, top_k <= %d)", T, E, top_k, kMaxExperts,
              kMaxTopK);
    return QL_ERR_ARG;
  }
  if (!counts || !offsets || !cursor || !active || !n_active || !n_tiles || (max_tiles > 0 && !tiles) ||
      (T > 0 && (!logits || !topk_idx || !topk_w || !row_token || !pair_row))) {
    set_error("ql_moe_route: null pointer");
    return QL_ERR_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  if (T <= kSmallTokens && (long)T * top_k <= kSmallPairs) {   // decode: one launch
    moe_route_small_kernel<<<1, 1024, 0, st>>>(logits, T, E, top_k, norm_topk_prob, tile_rows, topk_idx, topk_w, counts,
                                               offsets, active, n_active, tiles, n_tiles, max_tiles, row_token,
                                               pair_row);
    return cuda_status(cudaGetLastError(), "moe_route_small launch");
  }
  int rc = cuda_status(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, st), "ql_moe_route memset");
  if (rc) return rc;
  if (T > 0) {
    moe_topk_kernel<<<(T + 7) / 8, 256, 0, st>>>(logits, T, E, top_k, norm_topk_prob, topk_idx, topk_w, counts);
    if ((rc = cuda_status(cudaGetLastError(), "moe_topk launch"))) return rc;
  }
  moe_scan_kernel<<<1, (E + 31) & ~31, 0, st>>>(counts, E, tile_rows, offsets, cursor, active, n_active, tiles,
                                                n_tiles, max_tiles);
  if ((rc = cuda_status(cudaGetLastError(), "moe_scan launch"))) return rc;
  if (T > 0) {
    const int pairs = T * top_k;
    moe_scatter_kernel<<<(pairs + 255) / 256, 256, 0, st>>>(topk_idx, T, top_k, offsets, cursor, row_token,
                                                             pair_row);
    if ((rc = cuda_status(cudaGetLastError(), "moe_scatter launch"))) return rc;
  }
  return QL_OK;
}

extern "C" int ql_moe_group(const int32_t* ids, int n, int G, int tile_rows, int32_t* counts, int32_t* offsets,
                            int32_t* cursor, int32_t* active, int32_t* n_active, int32_t* tiles, int32_t* n_tiles,
                            int max_tiles, int32_t* row_src, int32_t* pos_of, void* stream) {
  if (n < 0 || G <= 0 || G > kMaxExperts || tile_rows <= 0 || max_tiles < 0) {
    set_error("ql_moe_group: bad sizes (n=%d G=%d; G <= %d)", n, G, kMaxExperts);
    return QL_ERR_ARG;
  }
  if (!counts || !offsets || !cursor || !active || !n_active || !n_tiles || (max_tiles > 0 && !tiles) ||
      (n > 0 && (!ids || !row_src || !pos_of))) {
    set_error("ql_moe_group: null pointer");
    return QL_ERR_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int rc = cuda_status(cudaMemsetAsync(counts, 0, sizeof(int32_t) * G, st), "ql_moe_group memset");
  if (rc) return rc;
  if (n > 0) {
    moe_hist_kernel<<<(n + 255) / 256, 256, 0, st>>>(ids, n, counts);
    if ((rc = cuda_status(cudaGetLastError(), "moe_hist launch"))) return rc;
  }
  moe_scan_kernel<<<1, (G + 31) & ~31, 0, st>>>(counts, G, tile_rows, offsets, cursor, active, n_active, tiles,
                                                n_tiles, max_tiles);
  if ((rc = cuda_status(cudaGetLastError(), "moe_scan launch"))) return rc;
  if (n > 0) {
    moe_scatter_kernel<<<(n + 255) / 256, 256, 0, st>>>(ids, n, 1, offsets, cursor, row_src, pos_of);
    if ((rc = cuda_status(cudaGetLastError(), "moe_scatter launch"))) return rc;
  }
  return QL_OK;
}

extern "C" int ql_moe_act(const float* y, long P, int I, void* a, int a_dtype, void* stream) {
  if (P < 0 || I <= 0 || (P > 0 && (!y || !a)) || a_dtype < QL_F32 || a_dtype > QL_BF16) {
    set_error("ql_moe_act: bad arguments");
    return QL_ERR_ARG;
  }
  if (P == 0) return QL_OK;
  const long total = P * I;
  const long blocks = (total + 255) / 256;
  moe_act_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, (cudaStream_t)stream>>>(y, P, I, a,
                                                                                                     a_dtype);
  return cuda_status(cudaGetLastError(), "moe_act launch");
}

extern "C" int ql_moe_combine(const float* z, const int32_t* pair_row, const float* topk_w, int T, int top_k, int H,
                              const float* shared, long lds, const float* shared_gate, long ldg, void* out,
                              int out_dtype, long ldo, void* stream) {
  if (T < 0 || top_k <= 0 || H <= 0 || (T > 0 && (!z || !pair_row || !topk_w || !out)) || ldo < H ||
      out_dtype < QL_F32 || out_dtype > QL_BF16 || (shared && lds < H) || (shared_gate && (!shared || ldg < 1))) {
    set_error("ql_moe_combine: bad arguments");
    return QL_ERR_ARG;
  }
  if (T == 0) return QL_OK;
  const bool vec = H % 4 == 0 && (reinterpret_cast<uintptr_t>(z) & 15) == 0 &&
                   (!shared || (lds % 4 == 0 && (reinterpret_cast<uintptr_t>(shared) & 15) == 0));
  if (vec) {
    const int parts = (H / 4 + 255) / 256;
    if ((long)T * parts < 0x7fffffffL) {
      moe_combine4_kernel<<<(unsigned)(T * parts), 256, 0, (cudaStream_t)stream>>>(
          z, pair_row, topk_w, top_k, H, parts, shared, lds, shared_gate, ldg, out, out_dtype, ldo);
      return cuda_status(cudaGetLastError(), "moe_combine launch");
    }
  }
  const long total = (long)T * H;
  const long blocks = (total + 255) / 256;
  moe_combine_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, (cudaStream_t)stream>>>(
      z, pair_row, topk_w, T, top_k, H, shared, lds, shared_gate, ldg, out, out_dtype, ldo);
  return cuda_status(cudaGetLastError(), "moe_combine launch");
}

namespace ql {
int gptq_gemv_grouped(const void* x, int x_dtype, long ldx, const int32_t* x_rows, const int32_t* qweight,
                      const int32_t* qzeros, const void* scales, int sc_dtype, long qw_estride, long qz_estride,
                      long sc_estride, const int32_t* offsets, const int32_t* active, const int32_t* n_active,
                      int max_active, int rows_hint, void* out, int out_dtype, long ldo, int K, int N, int gs,
                      int bits, float zoff, cudaStream_t st, int glu);
int gptq_gemm_grouped(const void* x, int x_dtype, long ldx, const int32_t* row_map, int P, const int32_t* qweight,
                      const int32_t* qzeros, const void* scales, int sc_dtype, long qw_estride, long qz_estride,
                      long sc_estride, const int32_t* offsets, const int32_t* tiles, const int32_t* n_tiles,
                      int max_tiles, int tile_rows_n, int n_experts, void* out, int out_dtype, long ldo, int K,
                      int N, int gs, int bits, float zoff, void* workspace, size_t ws_bytes, cudaStream_t st,
                      int glu);
size_t gptq_gemm_workspace(int M, int K);
bool gptq_gemv_tma_grouped(const void* x, int x_dtype, long ldx, const int32_t* x_rows, const int32_t* qweight,
                           const int32_t* qzeros, const void* scales, int sc_dtype, int E, const int32_t* offsets,
                           const int32_t* tiles, const int32_t* n_tiles, int max_tiles, int tile_rows, void* out,
                           int out_dtype, long ldo, int K, int N, int gs, int bits, float zoff, cudaStream_t st,
                           int* rc, int glu);
}  // namespace ql

// True when a grouped call over P rows and E experts takes the tensor-core GEMM: the average
// active expert then holds enough rows to fill a good part of a 128-row tile.
static bool grouped_uses_gemm(long P, int E, int K, int gs) {
  static int min_avg = -1;
  if (min_avg < 0) min_avg = env_int("QL_MOE_GEMM_MIN_ROWS", 12);   // measured crossover: 16 rows already faster
  const long act = P < E ? P : E;
  return act > 0 && P >= (long)min_avg * act && K % 64 == 0 && (gs % 64 == 0 || gs == 32);
}

// Token-tile height of the grouped tensor-core GEMM for an average of `avg` rows per active
// expert. A tile dequantises its expert's weight tile once whatever its height, and its MMA work
// grows with the height, so the lowest tile that holds most experts' rows wins: 32 up to 32
// rows on average, 64 up to 80, else 128.
static int gemm_tile_rows(long P, int E) {
  static int forced = -1;
  if (forced < 0) forced = env_int("QL_MOE_GEMM_TILE", 0);
  if (forced == 32 || forced == 64 || forced == 128) return forced;
  const long act = P < E ? P : E;
  const long avg = act > 0 ? (P + act - 1) / act : 0;
  return avg <= 32 ? 32 : avg <= 80 ? 64 : 128;
}

static bool is_gemm_tile(int tile_rows) { return tile_rows == 32 || tile_rows == 64 || tile_rows == 128; }

extern "C" int ql_moe_tile_rows(long P, int E, int K, int gs, int max_rows_per_expert) {
  if (grouped_uses_gemm(P, E, K, gs)) return gemm_tile_rows(P, E);
  static int forced = -1;
  if (forced < 0) forced = env_int("QL_MOE_GEMV_TILE", 0);
  if (forced == 4 || forced == 8) return forced;
  // decode GEMV: tiles of about twice the average rows per active expert (an expert with more
  // rows takes several tiles, whose weight reads mostly hit L2), at most the bound on rows
  const long act = P < E ? P : E;
  const long avg2 = act > 0 ? 2 * ((P + act - 1) / act) : 0;
  const long rows = avg2 < max_rows_per_expert ? avg2 : max_rows_per_expert;
  return rows <= 4 ? 4 : 8;
}

extern "C" size_t ql_moe_grouped_workspace(long P, int E, int K, int gs) {
  return grouped_uses_gemm(P, E, K, gs) ? gptq_gemm_workspace((int)P, K) : 0;
}

static int grouped_matmul_impl(const void* x, int x_dtype, long ldx, const int32_t* row_token, long P,
                               const int32_t* qweight, const int32_t* qzeros, const void* scales, int scales_dtype,
                               int E, const int32_t* offsets, const int32_t* active, const int32_t* n_active,
                               const int32_t* tiles, const int32_t* n_tiles, int max_tiles, int tile_rows,
                               int max_rows_per_expert, void* out, int out_dtype, long ldo, int K, int N, int gs,
                               int bits, float zero_offset, void* workspace, size_t workspace_bytes, void* stream,
                               int glu) {
  if (bits != 4 && bits != 8) {
    set_error("ql_moe_grouped_matmul: bits must be 4 or 8 (got %d)", bits);
    return QL_ERR_UNSUPPORTED;
  }
  const int per = 32 / bits;
  if (P < 0 || P > 0x7fffffffL || E <= 0 || K <= 0 || N <= 0 || gs <= 0 || K % gs || gs % per || N % 8 ||
      ldx < (glu ? 2L * K : (long)K) || ldo < N || max_rows_per_expert < 0) {
    set_error("ql_moe_grouped_matmul: bad sizes (P=%ld E=%d K=%d N=%d gs=%d; N %% 8 == 0, gs | K)", P, E, K, N, gs);
    return QL_ERR_ARG;
  }
  if (gs % 32 != 0 || (zero_offset != 0.f && zero_offset != 1.f)) {
    set_error("ql_moe_grouped_matmul: gs %% 32 == 0 and zero_offset in {0, 1} are supported");
    return QL_ERR_UNSUPPORTED;
  }
  if ((x_dtype != QL_F32 && x_dtype != QL_F16 && x_dtype != QL_BF16) ||
      (out_dtype != QL_F32 && out_dtype != QL_F16 && out_dtype != QL_BF16) ||
      (scales_dtype != QL_F32 && scales_dtype != QL_F16 && scales_dtype != QL_BF16)) {
    set_error("ql_moe_grouped_matmul: unknown dtype code");
    return QL_ERR_ARG;
  }
  if (!qweight || !qzeros || !scales || !offsets || !active || !n_active || (P > 0 && (!x || !out))) {
    set_error("ql_moe_grouped_matmul: null pointer");
    return QL_ERR_ARG;
  }
  if ((reinterpret_cast<uintptr_t>(qweight) | reinterpret_cast<uintptr_t>(scales)) & 15) {
    set_error("ql_moe_grouped_matmul: qweight and scales must be 16-byte aligned");
    return QL_ERR_ALIGN;
  }
  if (P == 0) return QL_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const long qw_es = (long)(K / per) * N, qz_es = (long)(K / gs) * (N / per), sc_es = (long)(K / gs) * N;
  if (is_gemm_tile(tile_rows) && grouped_uses_gemm(P, E, K, gs)) {
    if (!tiles || !n_tiles || max_tiles <= 0) {
      set_error("ql_moe_grouped_matmul: the tensor-core path needs the routing tile table");
      return QL_ERR_ARG;
    }
    int rc = gptq_gemm_grouped(x, x_dtype, ldx, row_token, (int)P, qweight, qzeros, scales, scales_dtype, qw_es,
                               qz_es, sc_es, offsets, tiles, n_tiles, max_tiles, tile_rows, E, out, out_dtype, ldo,
                               K, N, gs, bits, zero_offset, workspace, workspace_bytes, st, glu);
    if (rc != QL_ERR_UNSUPPORTED) return rc;
  }
  const int max_active = (int)(P < E ? P : E);
  int trc = 0;
  if (gptq_gemv_tma_grouped(x, x_dtype, ldx, row_token, qweight, qzeros, scales, scales_dtype, E, offsets, tiles,
                            n_tiles, max_tiles, tile_rows, out, out_dtype, ldo, K, N, gs, bits, zero_offset, st,
                            &trc, glu))
    return trc;
  return gptq_gemv_grouped(x, x_dtype, ldx, row_token, qweight, qzeros, scales, scales_dtype, qw_es, qz_es, sc_es,
                           offsets, active, n_active, max_active, max_rows_per_expert, out, out_dtype, ldo, K, N, gs,
                           bits, zero_offset, st, glu);
}

extern "C" int ql_moe_grouped_matmul(const void* x, int x_dtype, long ldx, const int32_t* row_token, long P,
                                     const int32_t* qweight, const int32_t* qzeros, const void* scales,
                                     int scales_dtype, int E, const int32_t* offsets, const int32_t* active,
                                     const int32_t* n_active, const int32_t* tiles, const int32_t* n_tiles,
                                     int max_tiles, int tile_rows, int max_rows_per_expert, void* out, int out_dtype,
                                     long ldo, int K, int N, int gs, int bits, float zero_offset, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  return grouped_matmul_impl(x, x_dtype, ldx, row_token, P, qweight, qzeros, scales, scales_dtype, E, offsets, active,
                             n_active, tiles, n_tiles, max_tiles, tile_rows, max_rows_per_expert, out, out_dtype, ldo,
                             K, N, gs, bits, zero_offset, workspace, workspace_bytes, stream, 0);
}

extern "C" int ql_moe_grouped_matmul_swiglu(const void* y, int y_dtype, long ldy, long P, const int32_t* qweight,
                                            const int32_t* qzeros, const void* scales, int scales_dtype, int E,
                                            const int32_t* offsets, const int32_t* active, const int32_t* n_active,
                                            const int32_t* tiles, const int32_t* n_tiles, int max_tiles,
                                            int tile_rows, int max_rows_per_expert, void* out, int out_dtype,
                                            long ldo, int K, int N, int gs, int bits, float zero_offset,
                                            void* workspace, size_t workspace_bytes, void* stream) {
  return grouped_matmul_impl(y, y_dtype, ldy, nullptr, P, qweight, qzeros, scales, scales_dtype, E, offsets, active,
                             n_active, tiles, n_tiles, max_tiles, tile_rows, max_rows_per_expert, out, out_dtype, ldo,
                             K, N, gs, bits, zero_offset, workspace, workspace_bytes, stream, K);
}
