// Device helpers shared by the two decode-GEMV kernels (register-fed and TMA-fed): loading
// activations, and staging them as power-of-two-scaled fp16 in the order the nibble unpack
// produces, together with the per-group sums that fold the zero point into the partial sums.
#pragma once

#include "ql_common.cuh"

namespace ql {

// Options of the fused decode-step GEMV (ql_gptq_matmul_fused): RMSNorm weight / eps folded into
// the activation staging, SwiGLU of [gate | up] rows (glu = K), and a residual added to the output.
struct GemvFused {
  const float* norm_w;
  float norm_eps;
  int glu;
  const float* res;
  long ldres;
};

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
// With a.nw (RMSNorm folded into the load) each value is multiplied by the token's factor
// a.nr[m] = 1 / sqrt(mean(x^2) + eps) and by the norm weight of its K index.
template <class Args>
__device__ __forceinline__ void load_x8(const Args& a, int m, int k, float (&v)[8]) {
  if (a.glu) {
    const long base = (long)(a.x_rows ? a.x_rows[m] : m) * a.ldx;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int src = a.x_perm ? a.x_perm[k + j] : k + j;
      v[j] = swiglu(load_as_float(a.x, a.x_dtype, base + src), load_as_float(a.x, a.x_dtype, base + a.glu + src));
    }
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
    if (a.nw) {
      const float r = a.nr[m];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = v[j] * r * a.nw[k + j];
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int src = a.x_perm ? a.x_perm[k + j] : k + j;
      v[j] = load_as_float(a.x, a.x_dtype, base + src);
      if (a.nw) v[j] = v[j] * a.nr[m] * a.nw[src];
    }
  }
}

// Sum of squares of token row m's K values of x (any order), reduced over the calling threads'
// warp (each lane covers a strided share). x_rows / x_perm / glu are not involved.
template <class Args>
__device__ __forceinline__ float row_sumsq_part(const Args& a, int m, int K, int part, int nparts) {
  float s = 0.f;
  const long base = (long)m * a.ldx;
  for (int k = part; k < K; k += nparts) {
    const float v = load_as_float(a.x, a.x_dtype, base + k);
    s = fmaf(v, v, s);
  }
  return s;
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

// ---------------------------------------------------------------------------------------
// Integer staging of activations for the integer-MMA GEMVs (u8 weights x s8 activation bytes)
// ---------------------------------------------------------------------------------------
// Every exponent group of EG consecutive values of one token (the quantisation group, or the
// Q4_K super-block) gets its own power of two: e such that max|x| * 2^-e lies in [2^21, 2^22),
// and each value becomes the integer v = rint(x * 2^-e), |v| <= 2^22 (23 bits: an element 1000x
// below its group's maximum still keeps 13 significant bits). v is split into three signed
// bytes, v = 2^16 b2 + 2^8 b1 + b0, which take MMA columns 4u, 4u + 1 and 4u + 3 of the token
// (u = its place in the n8 tile); column 4u + 2 is zero. With v1 = 2^8 b2 + b1 (|v1| <= 2^14)
// the MMA lane that owns the column pair (b2, b1) forms the exact int32 dot product with v1 as
// 256 D[4u] + D[4u + 1], and the lane that owns (0, b0) the one with b0 the same way; both
// lanes fold their group into fp32 with the factor 2^e (times 2^8 for the v1 lane, applied once
// at the end), and the two lanes' sums are added when the kernel finishes.
//
// B operand layout: the MMA n8 tile holds two tokens (columns 4u .. 4u + 3 for token u of the
// tile); in memory only the three used slots are stored, slot 3m + P (P = 0, 1, 2 for b2, b1, b0)
// of row (step, t), rows xb3_slots(M) slots apart.
// Slots per B row for m tokens: 3m rounded up to 4 (mod 8), which makes consecutive rows start 8
// or 24 banks apart, so the 8-byte loads of one half-warp (one token's three slots, four rows)
// are conflict-free.
__host__ __device__ constexpr int xb3_slots(int m) { return ((3 * m + 3) & ~7) + 4; }

// |bits| of the largest |x| of a chunk, compared as integers: NaN patterns sort above inf.
__device__ __forceinline__ uint32_t abs_bits_max(const float (&v)[8]) {
  uint32_t mb = 0u;
#pragma unroll
  for (int j = 0; j < 8; ++j) mb = max(mb, __float_as_uint(v[j]) & 0x7fffffffu);
  return mb;
}

// Exponent of a group whose largest |x| has bit pattern mb (finite): max|x| * 2^-e < 2^22,
// clamped below so that 2^-e stays a normal float (groups of values below 2^-105 keep fewer bits).
__device__ __forceinline__ int stage_exponent_i23(uint32_t mb) {
  if (mb == 0u) return 0;
  const int e = (int)(mb >> 23) - 127 - 21;
  return e < -126 ? -126 : e;
}

// Split 8 values (scaled by s) into the three byte planes, packed in MMA register order (BITS 4:
// even K offsets -> register 0, odd -> register 1, byte j / 2; BITS 8: values 0-3 -> register 0,
// 4-7 -> register 1, byte j % 4), and the chunk's sums of v1 and b0.
template <int BITS>
__device__ __forceinline__ void split3(const float (&v)[8], float s, uint32_t (&pl)[3][2], int& s1, int& s0) {
#pragma unroll
  for (int P = 0; P < 3; ++P) pl[P][0] = pl[P][1] = 0u;
  s1 = s0 = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int q = __float2int_rn(v[j] * s);
    const int b0 = (q << 24) >> 24;          // signed low byte
    const int q1 = (q - b0) >> 8;            // exact
    const int b1 = (q1 << 24) >> 24;
    const int b2 = (q1 - b1) >> 8;
    s1 += q1;
    s0 += b0;
    const int reg = BITS == 4 ? (j & 1) : (j >> 2);
    const int sh = 8 * (BITS == 4 ? (j >> 1) : (j & 3));
    pl[0][reg] |= (uint32_t)(b2 & 0xff) << sh;
    pl[1][reg] |= (uint32_t)(b1 & 0xff) << sh;
    pl[2][reg] |= (uint32_t)(b0 & 0xff) << sh;
  }
}

// Store the planes of chunk kc (8 values) of token m into the B layout. BITS 4: an int4 packed
// row r (K 8r .. 8r+7) is lane (r % 4)'s B registers of step r / 4 (even offsets -> MMA k 4t + i,
// odd -> 16 + 4t + i). BITS 8 (int8 weights, Q4_K bytes): packed rows 8s + t and 8s + 4 + t are
// lane t's two registers of step s; a chunk is rows 2kc and 2kc + 1.
template <int BITS>
__device__ __forceinline__ void put3(const uint32_t (&pl)[3][2], int m, int kc, int sstride, uint2* xb) {
  if constexpr (BITS == 4) {
    uint2* dst = xb + ((kc >> 2) * 4 + (kc & 3)) * sstride + 3 * m;
#pragma unroll
    for (int P = 0; P < 3; ++P) dst[P] = make_uint2(pl[P][0], pl[P][1]);
  } else {
    const int r0 = 2 * kc, s8 = r0 >> 3, j = r0 & 7, half = j >> 2, t0 = j & 3;
    uint32_t* d0 = reinterpret_cast<uint32_t*>(xb + (s8 * 4 + t0) * sstride + 3 * m) + half;
    uint32_t* d1 = reinterpret_cast<uint32_t*>(xb + (s8 * 4 + t0 + 1) * sstride + 3 * m) + half;
#pragma unroll
    for (int P = 0; P < 3; ++P) {
      d0[2 * P] = pl[P][0];
      d1[2 * P] = pl[P][1];
    }
  }
}

// One chunk (8 values of token m at chunk kc of the slice) of a warp that covers whole exponent
// groups: the group's exponent from a shuffle maximum over its EG / 8 lanes, the planes, and
// the group sums over SG / 8 lanes. `live` lanes store (put3, then sums(m, kc / (SG / 8), S1,
// S0) and expo(m, kc / (EG / 8), fe) from the first lane of each group); the others only take
// part in the shuffles. fe = 2^e, or NaN for a group holding inf / nan.
template <int BITS, int SG, int EG, class SumFn, class ExpFn>
__device__ __forceinline__ void stage_chunk3(const float (&v)[8], bool live, int m, int kc, int sstride, uint2* xb,
                                             SumFn& sums, ExpFn& expo) {
  constexpr int SSEG = SG / 8, ESEG = EG / 8;
  static_assert(ESEG >= SSEG && ESEG <= 32 && (ESEG & (ESEG - 1)) == 0, "exponent groups of 8 to 256 values");
  uint32_t mb = abs_bits_max(v);
#pragma unroll
  for (int o = ESEG / 2; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
  const bool finite = mb < 0x7f800000u;
  const int e = finite ? stage_exponent_i23(mb) : 0;
  uint32_t pl[3][2];
  int s1, s0;
  split3<BITS>(v, finite ? exp2i(-e) : 0.f, pl, s1, s0);
#pragma unroll
  for (int o = SSEG / 2; o > 0; o >>= 1) {
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s0 += __shfl_xor_sync(0xffffffffu, s0, o);
  }
  if (live) {
    put3<BITS>(pl, m, kc, sstride, xb);
    if (kc % SSEG == 0) sums(m, kc / SSEG, s1, s0);
    if (kc % ESEG == 0) expo(m, kc / ESEG, finite ? exp2i(e) : __int_as_float(0x7fc00000));
  }
}

// Stage x[:, kbase : kbase + klen] for M tokens (rows of `a`) into the three-plane B layout in
// shared memory, rows sstride slots apart (klen a multiple of EG). Every warp takes 32
// consecutive chunks of one token, so groups never straddle warps.
// NAMED: synchronise only the nthr participating threads with named barrier 1 (the TMA-fed
// kernels keep their producer warp out of the staging); otherwise __syncthreads.
template <int BITS, int SG, int EG, bool NAMED, class Args, class SumFn, class ExpFn>
__device__ void stage_x3(const Args& a, int kbase, int klen, int sstride, uint2* xb, SumFn sums, ExpFn expo, int tid,
                         int nthr) {
  constexpr int CH = 4;   // chunks a thread loads before converting (memory-level parallelism)
  const int M = a.M;
  const int cpr = klen / 8;
  const int nchunk = M * cpr;
  for (int base = 0; base < nchunk; base += CH * nthr) {
    float v[CH][8];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int idx = base + c * nthr + tid;
      if (idx < nchunk) {
        const int m = M == 1 ? 0 : idx / cpr;
        load_x8(a, m, kbase + (idx - m * cpr) * 8, v[c]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[c][j] = 0.f;
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int idx = base + c * nthr + tid;
      if (base + c * nthr + (tid & ~31) < nchunk) {   // warp-uniform: the warp's groups
        const int m = M == 1 ? 0 : idx / cpr;
        stage_chunk3<BITS, SG, EG>(v[c], idx < nchunk, m, idx - m * cpr, sstride, xb, sums, expo);
      }
    }
  }
  if constexpr (NAMED) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
  } else {
    __syncthreads();
  }
}

}  // namespace gemv

namespace {
// Activations staged once in global memory for the TMA-fed GEMVs of more than 4 tokens, so no
// CTA stages them itself. Tokens go in chunks of MAXM; chunk c at xg + c * chunk_bytes holds the
// B operand of all K (rows of xb3_slots(MAXM) slots) and, at sum_off, per stage-contiguous sums:
//   LAYOUT 0 (GPTQ, SG = EG = the group): group g at ints g * 3 * MAXM: [S1 | S0 | fe bits][MAXM]
//   LAYOUT 1 (Q4_K, SG = 32, EG = 256): super-block b at ints b * q4k_sum_ints(MAXM): sub-block
//            j's [S1 | S0][MAXM] at (2 j) * MAXM, then fe bits [MAXM] at 16 * MAXM (each
//            super-block's record padded to 128 bytes, so ring stages stay 128-byte aligned)
// One CTA of 256 threads per token row.
__host__ __device__ constexpr int q4k_sum_ints(int maxm) { return (17 * maxm + 31) & ~31; }

template <int BITS, int SG, int EG, int MAXM, int LAYOUT, class Args>
__global__ void __launch_bounds__(256) prestage_x3_kernel(const Args a, int K, uint8_t* __restrict__ xg,
                                                          long chunk_bytes, long sum_off) {
  constexpr int SS = gemv::xb3_slots(MAXM);
  const int m = blockIdx.x, c = m / MAXM, mm = m - c * MAXM;
  const int tid = threadIdx.x;
  const int cpr = K / 8;
  __shared__ float s_red[8];
  __shared__ float s_nr[1];
  Args an = a;   // this CTA's row: x from row m on, token index 0
  an.x = reinterpret_cast<const char*>(a.x) + (size_t)m * a.ldx * (a.x_dtype == QL_F32 ? 4 : 2);
  if (a.nw) {
    // RMSNorm folded into the staging: the row's factor over all K, then x * r * w on load
    float ss = gemv::row_sumsq_part(an, 0, K, tid, 256);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) s_red[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int w = 0; w < 8; ++w) t += s_red[w];
      s_nr[0] = rsqrtf(t / (float)K + a.norm_eps);
    }
    __syncthreads();
    an.nr = s_nr;
  }
  uint2* xb = reinterpret_cast<uint2*>(xg + (long)c * chunk_bytes);
  int* sm = reinterpret_cast<int*>(xg + (long)c * chunk_bytes + sum_off);
  auto sums = [&](int, int g, int s1, int s0) {
    if constexpr (LAYOUT == 0) {
      sm[(g * 3 + 0) * MAXM + mm] = s1;
      sm[(g * 3 + 1) * MAXM + mm] = s0;
    } else {
      const int b = g >> 3, j = g & 7;
      sm[b * q4k_sum_ints(MAXM) + (2 * j) * MAXM + mm] = s1;
      sm[b * q4k_sum_ints(MAXM) + (2 * j + 1) * MAXM + mm] = s0;
    }
  };
  auto expo = [&](int, int g, float fe) {
    if constexpr (LAYOUT == 0)
      sm[(g * 3 + 2) * MAXM + mm] = __float_as_int(fe);
    else
      sm[g * q4k_sum_ints(MAXM) + 16 * MAXM + mm] = __float_as_int(fe);
  };
  for (int base = 0; base < cpr; base += 256) {   // cpr is a multiple of 16 (32 for Q4_K)
    const int kc = base + tid;
    if (base + (tid & ~31) < cpr) {
      float v[8];
      if (kc < cpr) {
        gemv::load_x8(an, 0, kc * 8, v);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.f;
      }
      gemv::stage_chunk3<BITS, SG, EG>(v, kc < cpr, mm, kc, SS, xb, sums, expo);
    }
  }
}
}  // namespace
}  // namespace ql
