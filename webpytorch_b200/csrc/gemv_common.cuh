// Device helpers shared by the two decode-GEMV kernels (register-fed and TMA-fed): loading
// activations, and staging them as power-of-two-scaled fp16 in the order the nibble unpack
// produces, together with the per-group sums that fold the zero point into the partial sums.
#pragma once

#include "ql_common.cuh"

namespace ql {
namespace gemv {

// Position of value j of a packed word inside the fp16 staging of x. The register unpack
// pairs value j with value j + per/2 in one half2, so x is stored in the same pair order.
template <int PER>
__device__ __forceinline__ int stage_pos(int j) {
  return (j % (PER / 2)) * 2 + j / (PER / 2);
}
// the same inside an 8-value chunk (one int4 word, or two int8 words)
template <int PER>
__device__ __forceinline__ int chunk_pos(int j) {
  return (j / PER) * PER + stage_pos<PER>(j % PER);
}

// silu(g) * u, as the MoE act kernel computes it (silu(v) = v / (1 + e^-v))
__device__ __forceinline__ float swiglu(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// 8 consecutive activations x[m, k .. k+7] (through x_perm when set) as floats. With a.glu > 0
// a row holds [gate | up] halves a.glu elements apart and the activation is silu(gate) * up.
template <class Args>
__device__ __forceinline__ void load_x8(const Args& a, int m, int k, float (&v)[8]) {
  if (a.glu) {
    const long base = (long)(a.x_rows ? a.x_rows[m] : m) * a.ldx;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = swiglu(load_as_float(a.x, a.x_dtype, base + k + j), load_as_float(a.x, a.x_dtype, base + a.glu + k + j));
    return;
  }
  const long base = (long)(a.x_rows ? a.x_rows[m] : m) * a.ldx;   // x_rows: gather of token rows
  if (a.x_perm == nullptr && a.x_vec) {
    if (a.x_dtype == QL_F16) {
      const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(a.x) + base + k);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(u32_as_h2(w[i]));
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else if (a.x_dtype == QL_BF16) {
      const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.x) + base + k);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    } else {
      const float4 f0 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + base + k);
      const float4 f1 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + base + k + 4);
      v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
      v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int src = a.x_perm ? a.x_perm[k + j] : k + j;
      v[j] = load_as_float(a.x, a.x_dtype, base + src);
    }
  }
}

// Stage x[:, kbase : kbase + klen] for M tokens into shared memory as power-of-two-scaled
// fp16 in unpack order, and the per-(token, group) sums the folded zero point needs.
//
// The unpack feeds the MMA "magic" values 1024 + q (even K offsets of an int4 word, all of an
// int8 word) and 1024 + 16 q (odd K offsets of an int4 word) without subtracting anything, so
// the activations at odd int4 offsets are stored divided by 16 (exact). Then, per group,
//   MMA sum C = sum_k xs_k * magic_k = 1024 * A + sum_k x_k q_k,  A = sum_k xs_k (stored values)
//   sum_k x_k (q_k - z - off) = C - 1024 * A - (z + off) * S,    S = sum_k x_k (effective values)
// and gsum[m][g] = (A, S). sh_exp[m] = e with x_staged = x * 2^-e. sh_max must be zero and
// visible before the call.
//
// NAMED: synchronise only the nthr participating threads with named barrier 1 (the TMA-fed
// kernel keeps its producer warp out of the staging); otherwise __syncthreads.
template <int BITS, int GS, bool NAMED, class Args>
__device__ void stage_x(const Args& a, int kbase, int klen, int gstride, __half* xs, float2* gsum, int* sh_exp,
                        unsigned* sh_max, int tid, int nthr) {
  constexpr int PER = 32 / BITS;
  constexpr int CH = 4;          // 8-value chunks a thread keeps in registers on the one-pass path
  constexpr int SEG = GS / 8;    // chunks per group (lanes reduced together)
  const int M = a.M;
  auto sync = [&]() {
    if constexpr (NAMED) {
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    } else {
      __syncthreads();
    }
  };
  const int cpr = klen / 8;
  const int nchunk = M * cpr;
  auto store_chunk = [&](int idx, const float (&v)[8]) {
    const int m = idx / cpr, kc = idx - m * cpr;
    const float s = exp2i(-sh_exp[m]);
    __align__(16) __half h[8];
    float sa = 0.f, ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool hi = (BITS == 4) && (j & 1);
      const __half q = __float2half_rn(v[j] * s * (hi ? 0.0625f : 1.f));
      const float f = __half2float(q);
      sa += f;
      ss += hi ? 16.f * f : f;
      h[chunk_pos<PER>(j)] = q;
    }
    *reinterpret_cast<uint4*>(xs + (long)m * klen + kc * 8) = *reinterpret_cast<uint4*>(h);
    // the SEG chunks of one group sit in SEG consecutive lanes
#pragma unroll
    for (int o = SEG / 2; o > 0; o >>= 1) {
      sa += __shfl_xor_sync(0xffffffffu, sa, o);
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
    }
    if ((kc % SEG) == 0) gsum[m * gstride + kc / SEG] = make_float2(sa, ss);
  };
  if (nchunk <= nthr * CH) {
    float v[CH][8];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int idx = tid + c * nthr;
      if (idx < nchunk) {
        const int m = idx / cpr;
        load_x8(a, m, kbase + (idx - m * cpr) * 8, v[c]);
      }
    }
    // per-token maxima: reduce across the warp first when the whole warp is on one token
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int idx = tid + c * nthr;
      float mx = 0.f;
      if (idx < nchunk) {
#pragma unroll
        for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(v[c][j]));
      }
      const int base_idx = tid - (tid & 31) + c * nthr;
      const bool uniform = (cpr % 32 == 0) && base_idx < nchunk;
      if (uniform) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((tid & 31) == 0) atomicMax(&sh_max[base_idx / cpr], __float_as_uint(mx));
      } else if (idx < nchunk) {
        atomicMax(&sh_max[idx / cpr], __float_as_uint(mx));
      }
    }
    sync();
    if (tid < M) sh_exp[tid] = stage_exponent(__uint_as_float(sh_max[tid]));
    sync();
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int idx = tid + c * nthr;
      if (tid - (tid & 31) + c * nthr < nchunk) {   // warp-uniform: whole groups per warp
        store_chunk(idx, v[c]);
      }
    }
  } else {
    for (int m = 0; m < M; ++m) {
      float mx = 0.f;
      for (int kc = tid; kc < cpr; kc += nthr) {
        float v[8];
        load_x8(a, m, kbase + kc * 8, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(v[j]));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if ((tid & 31) == 0) atomicMax(&sh_max[m], __float_as_uint(mx));
    }
    sync();
    if (tid < M) sh_exp[tid] = stage_exponent(__uint_as_float(sh_max[tid]));
    sync();
    for (int base = 0; base < nchunk; base += nthr) {
      const int idx = base + tid;
      if (base + (tid - (tid & 31)) < nchunk) {      // warp-uniform
        float v[8];
        const int m = idx / cpr;
        load_x8(a, m, kbase + (idx - m * cpr) * 8, v);
        store_chunk(idx, v);
      }
    }
  }
  sync();
}

// Layout of the staged B operand: row (step, t) holds sstride slots (uint2 each). With the
// swizzle (SWZ, kernels of more than 4 tokens) slot s of row t is stored at s ^ xb_swz(sstride,
// t) and rows are rounded up to 8 slots: a warp's 64-bit loads of one step read rows t = 0..3,
// 4 slots each per half-warp, and the swizzle places the 4 rows 8 banks apart. Without it
// (up to 4 tokens) rows are 2M slots, unpadded.
__host__ __device__ constexpr int xb_slots(int slots) { return slots <= 4 ? slots : (slots + 7) & ~7; }
__host__ __device__ __forceinline__ int xb_swz(int sstride, int t) {
  return sstride <= 4 ? 0 : (sstride % 16 == 0 ? 4 * t : 4 * (t >> 1));
}

// Stage one 8-value chunk (chunk kc of a token's slice, scaled by s) of token m into the B
// operand layout described below; returns the chunk's sum of staged integers.
template <int BITS, bool SWZ>
__device__ __forceinline__ int put_chunk_i8(const float (&v)[8], float s, int m, int kc, int sstride, uint2* xb) {
  uint32_t hi[2] = {0u, 0u}, lo[2] = {0u, 0u};
  int sum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int q = __float2int_rn(v[j] * s);
    const int l = (int)(int8_t)(q & 0xff);
    const int h = (q - l) >> 8;
    sum += q;
    // int4: even offsets -> register 0, odd -> register 1; int8: first row -> 0, second -> 1
    const int reg = BITS == 4 ? (j & 1) : (j >> 2);
    const int byte = BITS == 4 ? (j >> 1) : (j & 3);
    hi[reg] |= (uint32_t)(h & 0xff) << (8 * byte);
    lo[reg] |= (uint32_t)(l & 0xff) << (8 * byte);
  }
  if constexpr (BITS == 4) {
    const int s4 = kc >> 2, t = kc & 3;
    uint2* dst = xb + (s4 * 4 + t) * sstride + (SWZ ? (2 * m) ^ xb_swz(sstride, t) : 2 * m);
    dst[0] = make_uint2(hi[0], hi[1]);
    dst[1] = make_uint2(lo[0], lo[1]);
  } else {
    const int r0 = 2 * kc;                // rows r0, r0 + 1 of the same half of a step
    const int s8 = r0 >> 3, j = r0 & 7;
    const int half = j >> 2, t0 = j & 3;
    const int c0 = SWZ ? (2 * m) ^ xb_swz(sstride, t0) : 2 * m;
    const int c1 = SWZ ? (2 * m) ^ xb_swz(sstride, t0 + 1) : 2 * m;
    uint32_t* d0 = reinterpret_cast<uint32_t*>(xb + (s8 * 4 + t0) * sstride + c0) + half;
    uint32_t* d1 = reinterpret_cast<uint32_t*>(xb + (s8 * 4 + t0 + 1) * sstride + c1) + half;
    d0[0] = hi[0];
    d0[2] = lo[0];
    d1[0] = hi[1];
    d1[2] = lo[1];
  }
  return sum;
}

// Stage x[:, kbase : kbase + klen] for M <= 16 tokens as the B operand of the integer MMA
// (mma.m16n8k32, A = u8 weights, B = s8 activations):
//   * each token row is scaled by an exact power of two, v = rint(x * 2^-e) with |v| <= 2^14
//     (sh_exp[m] = e), and split into two signed bytes v = 256 * hi + lo, which become two
//     MMA columns ("slots" 2m and 2m + 1) so that one MMA yields both partial dot products;
//   * the MMA K order follows the weight unpack. An int4 packed row r (K = 8r .. 8r+7) is
//     unpacked into bytes of even offsets (MMA k 4t + i <- K 8r + 2i) and odd offsets (MMA k
//     16 + 4t + i <- K 8r + 2i + 1), lane t of a 32-K step taking row 4s + t. An int8 packed row
//     (K = 4r .. 4r+3) is a register as it is: rows 8s + t and 8s + 4 + t feed MMA k 4t + i and
//     16 + 4t + i;
//   * xb[(s * 4 + t) * sstride + slot'] holds lane t's two B registers of step s for that slot
//     (slot' = slot ^ xb_swz(sstride, t) and sstride = xb_slots(2M) with SWZ, else slot and 2M);
//   * gsum[m * gstride + g] = sum of v over group g (exact integers), for the zero point.
// sh_max must be zero and visible before the call; sh_exp is valid after it returns.
template <int BITS, int GS, bool NAMED, bool SWZ, class Args>
__device__ void stage_x_i8(const Args& a, int kbase, int klen, int gstride, int sstride, uint2* xb, int* gsum,
                           int* sh_exp, unsigned* sh_max, int tid, int nthr) {
  constexpr int CH = 4;          // 8-value chunks a thread keeps in registers on the one-pass path
  constexpr int SEG = GS / 8;    // chunks per group (lanes reduced together)
  const int M = a.M;
  auto sync = [&]() {
    if constexpr (NAMED) {
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    } else {
      __syncthreads();
    }
  };
  const int cpr = klen / 8;
  const int nchunk = M * cpr;
  auto store_chunk = [&](int idx, const float (&v)[8]) {
    const int m = M == 1 ? 0 : idx / cpr, kc = idx - m * cpr;
    const float s = exp2i(-stage_exponent_i15(__uint_as_float(sh_max[m])));
    int sum = put_chunk_i8<BITS, SWZ>(v, s, m, kc, sstride, xb);
    // the SEG chunks of one group sit in SEG consecutive lanes
#pragma unroll
    for (int o = SEG / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((kc % SEG) == 0) gsum[m * gstride + kc / SEG] = sum;
  };
  auto row_max = [&](int m, float mx) { atomicMax(&sh_max[m], __float_as_uint(mx)); };
  if (nchunk <= nthr * CH) {
    float v[CH][8];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int idx = tid + c * nthr;
      if (idx < nchunk) {
        const int m = M == 1 ? 0 : idx / cpr;
        load_x8(a, m, kbase + (idx - m * cpr) * 8, v[c]);
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int idx = tid + c * nthr;
      float mx = 0.f;
      if (idx < nchunk) {
#pragma unroll
        for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(v[c][j]));
        if (mx != mx) mx = __int_as_float(0x7f800000);   // NaN counts as non-finite
      }
      const int base_idx = tid - (tid & 31) + c * nthr;
      const bool uniform = (cpr % 32 == 0) && base_idx < nchunk;
      if (uniform) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((tid & 31) == 0) row_max(base_idx / cpr, mx);
      } else if (idx < nchunk) {
        row_max(idx / cpr, mx);
      }
    }
    sync();
    // every thread derives its row's exponent from the maxima; sh_exp is read only after the
    // final barrier
    if (tid < M) sh_exp[tid] = stage_exponent_i15(__uint_as_float(sh_max[tid]));
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int idx = tid + c * nthr;
      if (tid - (tid & 31) + c * nthr < nchunk) {   // warp-uniform: whole groups per warp
        float w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = idx < nchunk ? v[c][j] : 0.f;
        if (idx < nchunk) store_chunk(idx, w);
        else {
          int z = 0;   // keep the group-sum shuffles converged
#pragma unroll
          for (int o = SEG / 2; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        }
      }
    }
  } else {
    for (int m = 0; m < M; ++m) {
      float mx = 0.f;
      for (int kc = tid; kc < cpr; kc += nthr) {
        float v[8];
        load_x8(a, m, kbase + kc * 8, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(v[j]));
        if (mx != mx) mx = __int_as_float(0x7f800000);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if ((tid & 31) == 0) row_max(m, mx);
    }
    sync();
    if (tid < M) sh_exp[tid] = stage_exponent_i15(__uint_as_float(sh_max[tid]));
    for (int base = 0; base < nchunk; base += nthr) {
      const int idx = base + tid;
      if (base + (tid - (tid & 31)) < nchunk) {      // warp-uniform
        float v[8];
        if (idx < nchunk) {
          const int m = idx / cpr;
          load_x8(a, m, kbase + (idx - m * cpr) * 8, v);
          store_chunk(idx, v);
        } else {
          int z = 0;
#pragma unroll
          for (int o = SEG / 2; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        }
      }
    }
  }
  sync();
}

// Activations staged once in global memory for the TMA-fed GEMVs of more than 4 tokens, so no
// CTA stages them itself: tokens in chunks of MAXM, chunk c at xg + c * chunk_bytes holding the
// B operand of all K (rows of xb_slots(2 MAXM) slots, swizzled, as stage_x_i8 with SWZ) and, at
// sum_off, the group sums as [group][MAXM]. xe[m] = the token's exponent e (x = v * 2^e), or
// kNonFinite for a row with inf / nan.
constexpr int kNonFinite = (int)0x80000000;

}  // namespace gemv

namespace {
// One CTA per token row (256 threads): the row's absolute maximum, then its 8-value chunks.
template <int BITS, int GS, int MAXM, class Args>
__global__ void __launch_bounds__(256) prestage_x_kernel(const Args a, int K, uint8_t* __restrict__ xg, long chunk_bytes,
                                                         long sum_off, int* __restrict__ xe) {
  constexpr int SEG = GS / 8;
  constexpr int SS = gemv::xb_slots(2 * MAXM);
  __shared__ float s_max[8];
  const int m = blockIdx.x, c = m / MAXM, mm = m - c * MAXM;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cpr = K / 8;
  float mx = 0.f;
  for (int kc = tid; kc < cpr; kc += 256) {
    float v[8];
    gemv::load_x8(a, m, kc * 8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(v[j]));
    if (mx != mx) mx = __int_as_float(0x7f800000);   // NaN counts as non-finite
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s_max[warp] = mx;
  __syncthreads();
  mx = s_max[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, s_max[w]);
  const int e = stage_exponent_i15(mx);
  if (tid == 0) xe[m] = mx < 3.0e38f ? e : gemv::kNonFinite;
  const float s = exp2i(-e);
  uint2* xb = reinterpret_cast<uint2*>(xg + (long)c * chunk_bytes);
  int* gsum = reinterpret_cast<int*>(xg + (long)c * chunk_bytes + sum_off);
  for (int base = 0; base < cpr; base += 256) {   // warp-uniform trip count (group shuffles)
    const int kc = base + tid;
    float v[8];
    if (kc < cpr) {
      gemv::load_x8(a, m, kc * 8, v);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    int sum = kc < cpr ? gemv::put_chunk_i8<BITS, true>(v, s, mm, kc, SS, xb) : 0;
#pragma unroll
    for (int o = SEG / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (kc < cpr && kc % SEG == 0) gsum[(kc / SEG) * MAXM + mm] = sum;
  }
}
}  // namespace
}  // namespace ql
