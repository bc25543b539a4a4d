// Shared device helpers for the SALT B200 kernels (sm_100a).
//
// Integer semantics follow the reference bit for bit:
//   * int32 arithmetic wraps (computed in uint32, like XLA's s32 ops);
//   * `>>` on int32 is an arithmetic shift (salt_core/quant/fixed_point.py:42-44);
//   * times are float32 holding integer ms; a queue Δt is a float32 subtraction truncated
//     toward zero (salt_core/connectivity/conv.py:119-125, salt_core/quant/codes.py:101);
//   * a dynamic gather index i maps to i + n when negative and is then clamped to [0, n-1]
//     (JAX out-of-bounds gather semantics, relied on by conv.py:160-162 when n_real = 0).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace salt {

constexpr float kPadTime = 1e12f;  // salt_core/stream.py:13 _PAD_TIME as float32

__device__ __forceinline__ int32_t wadd(int32_t a, int32_t b) {
  return (int32_t)((uint32_t)a + (uint32_t)b);
}
__device__ __forceinline__ int32_t wmul(int32_t a, int32_t b) {
  return (int32_t)((uint32_t)a * (uint32_t)b);
}
__host__ __device__ __forceinline__ int32_t floordiv(int32_t a, int32_t b) {
  int32_t q = a / b, r = a % b;
  return (r != 0 && ((r < 0) != (b < 0))) ? q - 1 : q;
}
__host__ __device__ __forceinline__ int32_t floormod(int32_t a, int32_t b) {
  int32_t r = a % b;
  return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}
__host__ __device__ __forceinline__ int64_t jax_index(int64_t i, int64_t n) {
  if (i < 0) i += n;
  if (i < 0) i = 0;
  if (i > n - 1) i = n - 1;
  return i;
}

// Fixed-point parameters of one layer, uniform across the launch.
struct QuantCfg {
  int32_t f_a, f_V, total_bits;  // total_bits = i_V + f_V
  int32_t round_half;            // 2^(f_a-1) in round mode with f_a > 0, else 0
  int32_t saturate;              // 0 wrap, 1 saturate
  int32_t lut_len;
};

// One event update (salt_core/quant/scan.py:22-52 process_event, with wide_mul_shift
// fixed_point.py:47-65 and fit_to_bits :68-90).  Returns the fitted (pre-reset) register
// value; `u` receives the unfitted value and `ovf` whether it left the register range.
__device__ __forceinline__ int32_t quant_step(int32_t v, int32_t a, bool is_identity, int32_t q,
                                              const QuantCfg& c, int32_t& u, bool& ovf) {
  int32_t hi = v >> c.f_a;
  int32_t lo = v & (int32_t)((1u << c.f_a) - 1u);
  int32_t dec = wadd(wmul(a, hi), wadd(wmul(a, lo), c.round_half) >> c.f_a);
  dec = is_identity ? v : dec;
  u = wadd(dec, wmul(q, (int32_t)(1u << c.f_V)));
  const int32_t half = (int32_t)(1u << (c.total_bits - 1));
  ovf = (u < -half) | (u >= half);
  int32_t w;
  if (c.saturate) {
    w = min(max(u, -half), half - 1);
  } else {
    const int sh = 32 - c.total_bits;  // two's-complement wrap into total_bits bits
    w = (int32_t)((uint32_t)u << sh) >> sh;
  }
  return w;
}

// The same update for the hot loops, with the identity step folded into the decay code: a
// step with Δt = 0 uses a = 2^f_a, for which the split multiply returns v exactly (hi * 2^f_a
// + lo, the rounding term is (2^f_a * lo + half) >> f_a = lo) for every register value of at
// most 30 bits; a decay code equal to 2^f_a likewise leaves v unchanged.  The overflow mode is a
// compile-time choice; ovf is "the fitted value differs from the unfitted one".
//
// WIDE computes the decay as one 64-bit product: with v = hi * 2^f_a + lo (0 <= lo < 2^f_a),
// a * hi + floor((a * lo + half) / 2^f_a) = floor((a * v + half) / 2^f_a) in the integers, so the
// two agree modulo 2^32 whenever the reference's int32 term a * lo + round_half does not wrap.
// That holds for every decay code in [0, 2^f_a] with f_a <= 15 (a * lo + half < 2^30), which is
// what a layer without needs_tail guarantees; other tables take the split form.
//
// Without FIT the fitted value is the unfitted one.  That is exact when the host has shown that
// no register can leave its range: with decay codes in [0, 2^f_a] a decay never grows |v|
// (floor((a*v + half) / 2^f_a) lies between 0 and v), so after n weighted steps
// |v| <= n * max|q| * 2^f_V, and n * 2^(q_bits - 1) < 2^(i_V - 1) keeps every value inside
// [-2^(i_V + f_V - 1), 2^(i_V + f_V - 1)), where wrap and saturate are both the identity.
template <bool SAT, bool WIDE = false, bool FIT = true>
__device__ __forceinline__ int32_t quant_step_a(int32_t v, int32_t a, int32_t q_shifted,
                                                int32_t f_a, int32_t lo_mask, int32_t round_half,
                                                int32_t half, int32_t wrap_shift, int32_t& u) {
  int32_t dec;
  if (WIDE)
    dec = (int32_t)(uint32_t)(uint64_t)(((int64_t)a * v + round_half) >> f_a);
  else
    dec = wadd(wmul(a, v >> f_a), wadd(wmul(a, v & lo_mask), round_half) >> f_a);
  u = wadd(dec, q_shifted);
  if (!FIT) return u;
  if (SAT) return min(max(u, -half), half - 1);
  return (int32_t)((uint32_t)u << wrap_shift) >> wrap_shift;
}

// Loop-invariant constants of quant_step_a.
struct StepConsts {
  int32_t f_a, f_V, lo_mask, round_half, half, wrap_shift, ident_a;
  __device__ __forceinline__ explicit StepConsts(const QuantCfg& c)
      : f_a(c.f_a), f_V(c.f_V), lo_mask((int32_t)((1u << c.f_a) - 1u)), round_half(c.round_half),
        half((int32_t)(1u << (c.total_bits - 1))), wrap_shift(32 - c.total_bits),
        ident_a((int32_t)(1u << c.f_a)) {}
  template <bool SAT, bool WIDE = false, bool FIT = true>
  __device__ __forceinline__ int32_t step(int32_t v, int32_t a, int32_t q, int32_t& u) const {
    return quant_step_a<SAT, WIDE, FIT>(v, a, wmul(q, (int32_t)(1u << f_V)), f_a, lo_mask,
                                        round_half, half, wrap_shift, u);
  }
};

// Step forms of the hot loops, chosen per layer on the host (step_form): the reference's split
// product; one 64-bit product (every decay code in [0, 2^f_a]); one 64-bit product and no fit
// (no register can leave its range either).
constexpr int kStepSplit = 0, kStepWide = 1, kStepWideNoFit = 2;

// apply_decay_table_int (salt_core/quant/codes.py:87-105) on an integer Δt.
__device__ __forceinline__ int32_t decay_code(int32_t dt, const int32_t* lut, int32_t lut_len) {
  if (lut_len <= 0) return 0;
  int32_t idx = min(max(wadd(dt, -1), 0), lut_len - 1);
  int32_t g = lut[idx];
  return dt > lut_len ? 0 : g;
}

__device__ __forceinline__ int32_t dt_from_times(float t, float t_prev) {
  return __float2int_rz(__fsub_rn(t, t_prev));  // float32 diff, astype(int32)
}

// Reads event `i` of a stream whose entries at or beyond `n_valid` are pads.  Internal streams
// written by this library do not materialise their pads ("virtual pads": time 1e12, src 0 as
// salt_core/stream.py:42-45 writes them); user-supplied streams carry their own pad values.
struct StreamView {
  const float* times;
  const int32_t* src;
  int32_t capacity;
  int32_t virtual_pads;
  __device__ __forceinline__ float time(int64_t row, int32_t i, int32_t n_valid) const {
    if (virtual_pads && i >= n_valid) return kPadTime;
    return times[row * capacity + i];
  }
  __device__ __forceinline__ int32_t source(int64_t row, int32_t i, int32_t n_valid) const {
    if (virtual_pads && i >= n_valid) return 0;
    return src[row * capacity + i];
  }
};

}  // namespace salt

namespace salt {

// Division of a non-negative int32 by a runtime constant d >= 1 with a precomputed multiplier
// (round-up method: q = (umulhi(x, m) + x) >> l, l = ceil(log2 d),
// m = floor(2^32 (2^l - d) / d) + 1; exact for 0 <= x < 2^31).  Built on the host.
struct FastDiv {
  uint32_t d, m, l;
  FastDiv() = default;
  __host__ explicit FastDiv(uint32_t divisor) : d(divisor) {
    l = 0;
    while ((1ull << l) < divisor) ++l;
    m = (uint32_t)((((1ull << 32) * ((1ull << l) - divisor)) / divisor) + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t x) const {
    return (__umulhi(x, m) + x) >> l;
  }
  __device__ __forceinline__ uint32_t mod(uint32_t x) const { return x - div(x) * d; }
};

}  // namespace salt
