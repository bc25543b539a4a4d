/*
 * CPU oracle for the SALT integer event-driven forward — TEST INFRASTRUCTURE ONLY.
 * See salt_oracle.h.  Every function cites the reference file:line it restates.
 * Parity pins: the reference's own known-answer tests, transcribed under tests/golden/.
 *
 * JAX semantics that the restatement reproduces on purpose:
 *   - int32 arithmetic wraps (two's complement); `>>` on int32 is arithmetic.
 *   - Python/JAX `//` and `%` on ints are floor division / floor modulo.
 *   - array indexing with a dynamic index first maps a negative index i to i + n and then
 *     clamps to [0, n-1] (out-of-bounds gathers clamp, they never fault).
 *   - times are float32; differences are float32 subtractions; `.astype(int32)` truncates.
 */
#include "salt_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#define SO_PAD_TIME ((float)1e12) /* stream.py:13 _PAD_TIME, stored as float32 */

static inline int32_t wadd(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }
static inline int32_t wmul(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); }
static inline int32_t floordiv(int32_t a, int32_t b) {
  int32_t q = a / b, r = a % b;
  return (r != 0 && ((r < 0) != (b < 0))) ? q - 1 : q;
}
static inline int32_t floormod(int32_t a, int32_t b) {
  int32_t r = a % b;
  return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}
/* JAX dynamic-index gather: negative index wraps once, then clamp into range. */
static inline int64_t jidx(int64_t i, int64_t n) {
  if (i < 0) i += n;
  if (i < 0) i = 0;
  if (i > n - 1) i = n - 1;
  return i;
}
static inline int32_t f32_to_i32(float x) { /* .astype(int32): truncation toward zero */
  if (!(x == x)) return 0;
  if (x >= 2147483647.0f) return 2147483647;
  if (x <= -2147483648.0f) return (int32_t)0x80000000u;
  return (int32_t)x;
}

/* fixed_point.py:32-44 round_shift */
int32_t so_round_shift(int32_t x, int32_t shift_bits, int32_t round_mode) {
  if (shift_bits == 0) return x;
  if (round_mode == SO_ROUND) x = wadd(x, (int32_t)(1u << (shift_bits - 1)));
  return x >> shift_bits;
}

/* fixed_point.py:47-65 wide_mul_shift */
int32_t so_wide_mul_shift(int32_t a, int32_t v, int32_t shift_bits, int32_t round_mode) {
  int32_t hi = v >> shift_bits;
  int32_t lo = v & (int32_t)((1u << shift_bits) - 1u);
  return wadd(wmul(a, hi), so_round_shift(wmul(a, lo), shift_bits, round_mode));
}

/* fixed_point.py:68-90 fit_to_bits */
int32_t so_fit_to_bits(int32_t x, int32_t total_bits, int32_t overflow_mode, int32_t *overflowed) {
  int32_t half = (int32_t)(1u << (total_bits - 1));
  *overflowed = (x < -half) || (x >= half);
  if (overflow_mode == SO_SATURATE) {
    if (x < -half) return -half;
    if (x > half - 1) return half - 1;
    return x;
  }
  int32_t masked = x & (int32_t)((1u << total_bits) - 1u);
  return masked >= half ? masked - (int32_t)(1u << total_bits) : masked;
}

/* quant/scan.py:22-52 process_event */
int32_t so_process_event(int32_t v0, int32_t a, int32_t is_identity, int32_t q, int32_t has_vth,
                         int32_t vth, int32_t f_a, int32_t f_V, int32_t i_V, int32_t round_mode,
                         int32_t overflow_mode, int32_t *is_spiked, int32_t *overflowed,
                         int32_t *v_unfitted) {
  int32_t decayed_active = so_wide_mul_shift(a, v0, f_a, round_mode);
  int32_t decayed = is_identity ? v0 : decayed_active;
  int32_t u = wadd(decayed, wmul(q, (int32_t)(1u << f_V)));
  int32_t fitted = so_fit_to_bits(u, i_V + f_V, overflow_mode, overflowed);
  *v_unfitted = u;
  if (!has_vth) {
    *is_spiked = 0;
    return fitted;
  }
  *is_spiked = fitted >= vth;
  return *is_spiked ? 0 : fitted;
}

/* quant/codes.py:87-105 apply_decay_table_int */
void so_apply_decay_table(const float *delta_t, int64_t n, const int32_t *lut, int32_t lut_len,
                          int32_t *a_int, uint8_t *is_identity) {
  for (int64_t i = 0; i < n; ++i) {
    int32_t dt = f32_to_i32(delta_t[i]);
    int32_t gathered = 0;
    if (lut_len > 0) {
      int32_t idx = dt - 1;
      if (idx < 0) idx = 0;
      if (idx > lut_len - 1) idx = lut_len - 1;
      gathered = lut[idx];
    }
    a_int[i] = dt > lut_len ? 0 : gathered;
    is_identity[i] = dt == 0;
  }
}

static void run_layer_traced(const int32_t *a_int, const uint8_t *is_identity,
                             const int32_t *q_int, const int32_t *vth, int32_t n, int32_t L,
                             int32_t f_a, int32_t f_V, int32_t i_V, int32_t round_mode,
                             int32_t overflow_mode, uint8_t *spike_mask, uint8_t *overflowed,
                             int32_t *v_final, int32_t *vmin, int32_t *vmax, int32_t *v_steps);

/* quant/scan.py:97-132 _run_layer_scan (trace=False): every one of the L columns is applied. */
void so_run_layer(const int32_t *a_int, const uint8_t *is_identity, const int32_t *q_int,
                  const int32_t *vth, int32_t n, int32_t L, int32_t f_a, int32_t f_V, int32_t i_V,
                  int32_t round_mode, int32_t overflow_mode, uint8_t *spike_mask,
                  uint8_t *overflowed, int32_t *v_final, int32_t *vmin, int32_t *vmax) {
  run_layer_traced(a_int, is_identity, q_int, vth, n, L, f_a, f_V, i_V, round_mode,
                   overflow_mode, spike_mask, overflowed, v_final, vmin, vmax, NULL);
}

/* _run_layer_scan with trace=True (quant/scan.py:83-94): also the register after each column. */
static void run_layer_traced(const int32_t *a_int, const uint8_t *is_identity,
                             const int32_t *q_int, const int32_t *vth, int32_t n, int32_t L,
                             int32_t f_a, int32_t f_V, int32_t i_V, int32_t round_mode,
                             int32_t overflow_mode, uint8_t *spike_mask, uint8_t *overflowed,
                             int32_t *v_final, int32_t *vmin, int32_t *vmax, int32_t *v_steps) {
  for (int32_t i = 0; i < n; ++i) {
    int32_t v = 0, lo = 0, hi = 0;
    for (int32_t t = 0; t < L; ++t) {
      int64_t e = (int64_t)i * L + t;
      int32_t spk, ovf, u;
      v = so_process_event(v, a_int[e], is_identity[e], q_int[e], vth != NULL,
                           vth ? vth[i] : 0, f_a, f_V, i_V, round_mode, overflow_mode, &spk, &ovf,
                           &u);
      if (u < lo) lo = u;
      if (u > hi) hi = u;
      if (spike_mask) spike_mask[e] = (uint8_t)spk;
      if (overflowed) overflowed[e] = (uint8_t)ovf;
      if (v_steps) v_steps[e] = v;
    }
    v_final[i] = v;
    vmin[i] = lo;
    vmax[i] = hi;
  }
}

/* connectivity/conv.py:15-29 _axis_candidates (one event, one axis). */
static void axis_candidates(int32_t i, int32_t K, int32_t S, int32_t P, int32_t N, int32_t O_max,
                            int32_t *o, uint8_t *valid) {
  int32_t o_min = floordiv(i + P - K + 1 + S - 1, S);
  int32_t upper = floordiv(i + P, S);
  for (int32_t r = 0; r < N; ++r) {
    o[r] = o_min + r;
    valid[r] = (o[r] <= upper) && (o[r] >= 0) && (o[r] < O_max);
  }
}

static int32_t conv_h_out(const so_conv_geom *g) { return (g->h_in + 2 * g->p - g->k) / g->s + 1; }
static int32_t conv_w_out(const so_conv_geom *g) { return (g->w_in + 2 * g->p - g->k) / g->s + 1; }

typedef struct {
  int32_t n, j;
} cand_t;

/* Stable sort of candidates by n (candidates are generated in j order, so this is the
 * reference's lexsort((j, n)) at conv.py:71).  Counting sort over n in [0, n_sp]. */
static void stable_sort_by_n(cand_t *c, int64_t C, int32_t n_buckets, cand_t *tmp) {
  int64_t *cnt = (int64_t *)calloc((size_t)n_buckets + 1, sizeof(int64_t));
  for (int64_t i = 0; i < C; ++i) cnt[c[i].n + 1]++;
  for (int32_t b = 0; b < n_buckets; ++b) cnt[b + 1] += cnt[b];
  for (int64_t i = 0; i < C; ++i) tmp[cnt[c[i].n]++] = c[i];
  memcpy(c, tmp, (size_t)C * sizeof(cand_t));
  free(cnt);
}

/* connectivity/conv.py:57-99 _compress_candidates.  lexsort((j, n)) is a stable sort by n of
 * candidates listed in j order; ties on (n, j) occur only among invalid candidates. */
int so_compress_candidates(const int32_t *n_flat, const int32_t *j_flat, int64_t C, int32_t n_sp,
                           int32_t L, int32_t n_events, int32_t *l2g, int32_t *n_real) {
  if (C < 0 || n_sp < 0 || L < 0) return -1;
  cand_t *c = (cand_t *)malloc(sizeof(cand_t) * (size_t)(C > 0 ? C : 1));
  cand_t *tmp = (cand_t *)malloc(sizeof(cand_t) * (size_t)(C > 0 ? C : 1));
  if (!c || !tmp) {
    free(c);
    free(tmp);
    return -3;
  }
  /* lexsort orders by n then by j: sort by j first (stable), then by n (stable) */
  for (int64_t i = 0; i < C; ++i) {
    c[i].n = n_flat[i] < n_sp ? n_flat[i] : n_sp; /* any n >= n_sp is the invalid bucket */
    c[i].j = j_flat[i];
  }
  /* stable order by j: candidates may be given in any order */
  for (int64_t w = 1; w < C; w *= 2) {
    for (int64_t lo = 0; lo < C; lo += 2 * w) {
      int64_t mid = lo + w < C ? lo + w : C, hi = lo + 2 * w < C ? lo + 2 * w : C;
      int64_t a = lo, b = mid, o = lo;
      while (a < mid && b < hi) tmp[o++] = c[b].j < c[a].j ? c[b++] : c[a++];
      while (a < mid) tmp[o++] = c[a++];
      while (b < hi) tmp[o++] = c[b++];
    }
    memcpy(c, tmp, sizeof(cand_t) * (size_t)C);
  }
  stable_sort_by_n(c, C, n_sp + 1, tmp);
  for (int64_t i = 0; i < (int64_t)n_sp * L; ++i) l2g[i] = n_events;
  memset(n_real, 0, sizeof(int32_t) * (size_t)n_sp);
  int64_t last_start = 0;
  for (int64_t i = 0; i < C; ++i) {
    if (i == 0 || c[i].n != c[i - 1].n) last_start = i;
    int64_t rank = i - last_start;
    if (c[i].n >= n_sp) continue; /* trash row */
    if (rank < L) l2g[(int64_t)c[i].n * L + rank] = c[i].j;
    if (rank + 1 > n_real[c[i].n]) n_real[c[i].n] = (int32_t)(rank + 1);
  }
  free(c);
  free(tmp);
  return 0;
}

/* connectivity/conv.py:102-125 _delta_t_three_regimes */
void so_delta_t_regimes(const float *t_gathered, const int32_t *n_real, float global_last,
                        int32_t n, int32_t L, float *delta_t) {
  for (int32_t i = 0; i < n; ++i) {
    const float *tg = t_gathered + (int64_t)i * L;
    int32_t lr = n_real[i] - 1;
    if (lr < 0) lr = 0;
    if (lr > L - 1) lr = L - 1;
    float catchup = global_last - tg[lr];
    float prev = 0.0f;
    for (int32_t col = 0; col < L; ++col) {
      float d = tg[col] - prev;
      prev = tg[col];
      delta_t[(int64_t)i * L + col] = col < n_real[i] ? d : (col == n_real[i] ? catchup : 0.0f);
    }
  }
}

/* connectivity/conv.py:128-172 build_conv_structure, with _compress_candidates (:57-99) and
 * _delta_t_three_regimes (:102-125). */
int so_conv_structure(const so_conv_geom *g, const float *times, const int32_t *src, int32_t E_len,
                      int32_t n_in, int32_t *l2g, int32_t *n_real, float *delta_t, int32_t *tap_c,
                      int32_t *tap_ky, int32_t *tap_kx) {
  const int32_t K = g->k, S = g->s, P = g->p, L = g->max_queue_len;
  const int32_t h_out = conv_h_out(g), w_out = conv_w_out(g), n_sp = h_out * w_out;
  const int32_t N = (K - 1) / S + 1, hw = g->h_in * g->w_in;
  if (E_len <= 0 || L <= 0 || n_sp <= 0) return -1;

  int32_t *ex = (int32_t *)malloc(sizeof(int32_t) * (size_t)E_len * 3);
  int32_t *ey = ex + E_len, *ec = ey + E_len;
  for (int32_t j = 0; j < E_len; ++j) { /* conv.py:32-43 unravel_conv_source */
    int32_t s = src[j];
    ec[j] = floordiv(s, hw);
    int32_t rem = floormod(s, hw);
    ey[j] = floordiv(rem, g->w_in);
    ex[j] = floormod(rem, g->w_in);
  }

  int64_t C = (int64_t)E_len * N * N;
  cand_t *cand = (cand_t *)malloc(sizeof(cand_t) * (size_t)C);
  cand_t *tmp = (cand_t *)malloc(sizeof(cand_t) * (size_t)C);
  if (!ex || !cand || !tmp) {
    free(ex);
    free(cand);
    free(tmp);
    return -3;
  }
  int32_t oy[64], ox[64];
  uint8_t vy[64], vx[64];
  if (N > 64) return -2;
  for (int32_t j = 0; j < E_len; ++j) {
    axis_candidates(ey[j], K, S, P, N, h_out, oy, vy);
    axis_candidates(ex[j], K, S, P, N, w_out, ox, vx);
    int real = j < n_in;
    for (int32_t a = 0; a < N; ++a)
      for (int32_t b = 0; b < N; ++b) {
        int64_t k = ((int64_t)j * N + a) * N + b;
        int valid = vy[a] && vx[b] && real;
        cand[k].n = valid ? oy[a] * w_out + ox[b] : n_sp;
        cand[k].j = j;
      }
  }
  free(tmp);
  {
    int32_t *nf = (int32_t *)malloc(sizeof(int32_t) * (size_t)C * 2);
    if (!nf) {
      free(ex);
      free(cand);
      return -3;
    }
    int32_t *jf = nf + C;
    for (int64_t i = 0; i < C; ++i) {
      nf[i] = cand[i].n;
      jf[i] = cand[i].j;
    }
    free(cand);
    int rc = so_compress_candidates(nf, jf, C, n_sp, L, E_len, l2g, n_real);
    free(nf);
    if (rc) {
      free(ex);
      return rc;
    }
  }

  /* conv.py:159-162: empty columns clamp to the last real event; gather semantics as JAX. */
  float global_last = times[jidx((int64_t)n_in - 1, E_len)];
  for (int32_t pos = 0; pos < n_sp; ++pos) {
    int32_t oyy = pos / w_out, oxx = pos % w_out;
    const int32_t *row = l2g + (int64_t)pos * L;
    float *dt = delta_t + (int64_t)pos * L;
    /* gathered times per column */
    int32_t nr = n_real[pos];
    int32_t last_real_col = nr - 1;
    if (last_real_col < 0) last_real_col = 0;
    if (last_real_col > L - 1) last_real_col = L - 1;
    int32_t ej_last = row[last_real_col] < n_in - 1 ? row[last_real_col] : n_in - 1;
    float t_last_real = times[jidx(ej_last, E_len)];
    float prev = 0.0f;
    for (int32_t col = 0; col < L; ++col) {
      int32_t ej = row[col] < n_in - 1 ? row[col] : n_in - 1;
      int64_t gi = jidx(ej, E_len);
      float tg = times[gi];
      float d_real = tg - prev;
      prev = tg;
      if (col < nr)
        dt[col] = d_real;
      else if (col == nr)
        dt[col] = global_last - t_last_real;
      else
        dt[col] = 0.0f;
      /* conv.py:164-171 taps, clipped into the kernel */
      int32_t ky = ey[gi] - oyy * S + P, kx = ex[gi] - oxx * S + P;
      tap_ky[(int64_t)pos * L + col] = ky < 0 ? 0 : (ky > K - 1 ? K - 1 : ky);
      tap_kx[(int64_t)pos * L + col] = kx < 0 ? 0 : (kx > K - 1 ? K - 1 : kx);
      tap_c[(int64_t)pos * L + col] = ec[gi];
    }
  }
  free(ex);
  return 0;
}

/* stream.py:49-64 _select_spikes + :84-100 / :67-81 + :24-46 _pack_stream. */
void so_extract_output_events(const uint8_t *mask, const int32_t *event_idx, int32_t n,
                              int32_t steps, const int32_t *l2g, int32_t l2g_rows, int32_t L,
                              const float *times, int32_t E_len, int32_t M, float *out_times,
                              int32_t *out_src, int32_t *n_real_out) {
  size_t cap = (size_t)(M > 0 ? M : 1);
  int32_t *nidx = (int32_t *)calloc(cap, sizeof(int32_t)); /* nonzero(..., fill_value=0) */
  int32_t *sidx = (int32_t *)calloc(cap, sizeof(int32_t));
  int64_t total = 0;
  for (int32_t i = 0; i < n; ++i)
    for (int32_t t = 0; t < steps; ++t)
      if (mask[(int64_t)i * steps + t]) {
        if (total < M) {
          nidx[total] = i;
          sidx[total] = t;
        }
        total++;
      }
  const int32_t nr = (int32_t)total;
  int32_t *key = (int32_t *)malloc(sizeof(int32_t) * cap);
  int32_t *gj = (int32_t *)malloc(sizeof(int32_t) * cap);
  for (int32_t k = 0; k < M; ++k) {
    /* queue column of the selected step (spike_event_idx[neuron, step]) */
    int32_t col = event_idx ? event_idx[(int64_t)nidx[k] * steps + sidx[k]] : sidx[k];
    int32_t g = col;
    if (l2g) { /* conv: local column -> global index via tile_channels(local_to_global_j) */
      int32_t c = col < L - 1 ? col : L - 1;
      g = l2g[(int64_t)(nidx[k] % l2g_rows) * L + c];
    }
    gj[k] = g;
    key[k] = k < nr ? g : E_len;
  }
  /* stable sort of 0..M-1 by key: jnp.lexsort on one key is stable */
  int32_t *order = (int32_t *)malloc(sizeof(int32_t) * cap);
  int32_t *tmpo = (int32_t *)malloc(sizeof(int32_t) * cap);
  for (int32_t k = 0; k < M; ++k) order[k] = k;
  for (int32_t width = 1; width < M; width *= 2) {
    for (int32_t lo = 0; lo < M; lo += 2 * width) {
      int32_t mid = lo + width < M ? lo + width : M, hi = lo + 2 * width < M ? lo + 2 * width : M;
      int32_t a = lo, b = mid, o = lo;
      while (a < mid && b < hi) tmpo[o++] = key[order[b]] < key[order[a]] ? order[b++] : order[a++];
      while (a < mid) tmpo[o++] = order[a++];
      while (b < hi) tmpo[o++] = order[b++];
    }
    memcpy(order, tmpo, sizeof(int32_t) * (size_t)M);
  }
  for (int32_t k = 0; k < M; ++k) {
    int32_t src_k = order[k];
    int real = src_k < nr;
    int32_t safe = gj[src_k] < E_len - 1 ? gj[src_k] : E_len - 1;
    out_times[k] = real ? times[jidx(safe, E_len)] : SO_PAD_TIME;
    out_src[k] = nidx[src_k];
  }
  *n_real_out = nr;
  free(nidx);
  free(sidx);
  free(key);
  free(gj);
  free(order);
  free(tmpo);
}

static void reduce_layer(so_layer_out *out, int32_t n, int32_t L, const uint8_t *ovf) {
  out->any_overflow = 0;
  for (int64_t e = 0; e < (int64_t)n * L; ++e)
    if (ovf[e]) {
      out->any_overflow = 1;
      break;
    }
  int32_t lo = out->vmin[0], hi = out->vmax[0];
  for (int32_t i = 1; i < n; ++i) {
    if (out->vmin[i] < lo) lo = out->vmin[i];
    if (out->vmax[i] > hi) hi = out->vmax[i];
  }
  out->vmin_all = lo;
  out->vmax_all = hi;
}

/* layers/conv.py:124-149 ConvLayer.forward with QuantBackend.scan (quant/backend.py:31-53). */
int so_conv_forward(const so_conv_geom *g, const so_quant_params *qp, const float *times,
                    const int32_t *src, int32_t E_len, int32_t n_in, so_layer_out *out) {
  const int32_t L = g->max_queue_len, h_out = conv_h_out(g), w_out = conv_w_out(g);
  const int32_t n_sp = h_out * w_out, OC = g->oc, n = OC * n_sp, K = g->k;
  if (h_out < 1 || w_out < 1 || L < 1) return -1;
  /* the dense (n, L) restatement needs n*L cells per array: refuse absurd capacities */
  if ((double)OC * n_sp * L > 4.0e9) return -4;
  size_t nl = (size_t)n_sp * L;
  int32_t *l2g = (int32_t *)malloc(sizeof(int32_t) * nl);
  int32_t *nreal = (int32_t *)malloc(sizeof(int32_t) * (size_t)n_sp);
  float *dt = (float *)malloc(sizeof(float) * nl);
  int32_t *tc = (int32_t *)malloc(sizeof(int32_t) * nl * 3);
  int32_t *tky = tc + nl, *tkx = tky + nl;
  int rc = so_conv_structure(g, times, src, E_len, n_in, l2g, nreal, dt, tc, tky, tkx);
  if (rc) return rc;

  /* neuron_delta_t = tile_channels(delta_t) (layers/conv.py:167-169); codes per connectivity/conv.py:210-219 */
  size_t NL = (size_t)n * L;
  int32_t *a = (int32_t *)malloc(sizeof(int32_t) * NL);
  uint8_t *isid = (uint8_t *)malloc(NL);
  int32_t *qi = (int32_t *)malloc(sizeof(int32_t) * NL);
  int32_t *a_sp = (int32_t *)malloc(sizeof(int32_t) * nl);
  uint8_t *id_sp = (uint8_t *)malloc(nl);
  so_apply_decay_table(dt, (int64_t)nl, qp->lut, qp->lut_len, a_sp, id_sp);
  for (int32_t o = 0; o < OC; ++o)
    for (int32_t pos = 0; pos < n_sp; ++pos)
      for (int32_t col = 0; col < L; ++col) {
        size_t e = ((size_t)o * n_sp + pos) * L + col, es = (size_t)pos * L + col;
        a[e] = a_sp[es];
        isid[e] = id_sp[es];
        int real = col < nreal[pos];
        int64_t c = jidx(tc[es], g->ic);
        int32_t qv = qp->q[(((int64_t)o * g->ic + c) * K + tky[es]) * K + tkx[es]];
        qi[e] = real ? qv : 0;
      }
  uint8_t *mask = out->spike_mask ? out->spike_mask : (uint8_t *)malloc(NL);
  uint8_t *ovf = out->overflowed ? out->overflowed : (uint8_t *)malloc(NL);
  run_layer_traced(a, isid, qi, qp->vth, n, L, qp->f_a, qp->f_V, qp->i_V, qp->round_mode,
                   qp->overflow_mode, mask, ovf, out->v_final, out->vmin, out->vmax,
                   out->v_steps);
  if (out->event_ms) /* trace.py:40-55 resolve_ms_conv with pointer = column */
    for (int32_t o = 0; o < OC; ++o)
      for (int32_t pos = 0; pos < n_sp; ++pos)
        for (int32_t col = 0; col < L; ++col) {
          int64_t j = l2g[(size_t)pos * L + col];
          if (j > E_len - 1) j = E_len - 1;
          out->event_ms[((size_t)o * n_sp + pos) * L + col] =
              col >= nreal[pos] ? (float)NAN : times[j];
        }
  so_extract_output_events(mask, NULL, n, L, l2g, n_sp, L, times, E_len, g->max_out_spikes,
                           out->out_times, out->out_src, &out->n_real_out);
  out->spike_count = out->n_real_out;
  int32_t mx = 0;
  for (int32_t pos = 0; pos < n_sp; ++pos)
    if (nreal[pos] > mx) mx = nreal[pos];
  out->needed_queue = mx + 1; /* layers/conv.py:137-141 */
  reduce_layer(out, n, L, ovf);
  out->fits = out->needed_queue <= L && out->n_real_out <= g->max_out_spikes &&
              0 <= g->max_extra_steps; /* capacity.py:60-63 */
  if (!out->spike_mask) free(mask);
  if (!out->overflowed) free(ovf);
  free(l2g);
  free(nreal);
  free(dt);
  free(tc);
  free(a);
  free(isid);
  free(qi);
  free(a_sp);
  free(id_sp);
  return 0;
}

/* layers/fc.py:84-101 FCLayer.forward with QuantBackend; structure per connectivity/fc.py:20-33,
 * codes per fc.py:54-61. */
int so_fc_forward(const so_fc_geom *g, const so_quant_params *qp, const float *times,
                  const int32_t *src, int32_t E_len, int32_t n_in, so_layer_out *out) {
  const int32_t n = g->n_out, L = E_len;
  if (E_len <= 0) return -1;
  float *dt = (float *)malloc(sizeof(float) * (size_t)L);
  float prev = 0.0f;
  for (int32_t j = 0; j < L; ++j) {
    float gap = times[j] - prev;
    prev = times[j];
    dt[j] = j < n_in ? gap : 0.0f;
  }
  int32_t *a1 = (int32_t *)malloc(sizeof(int32_t) * (size_t)L);
  uint8_t *id1 = (uint8_t *)malloc((size_t)L);
  so_apply_decay_table(dt, L, qp->lut, qp->lut_len, a1, id1);
  size_t NL = (size_t)n * L;
  int32_t *a = (int32_t *)malloc(sizeof(int32_t) * NL);
  uint8_t *isid = (uint8_t *)malloc(NL);
  int32_t *qi = (int32_t *)malloc(sizeof(int32_t) * NL);
  for (int32_t o = 0; o < n; ++o)
    for (int32_t j = 0; j < L; ++j) {
      size_t e = (size_t)o * L + j;
      a[e] = a1[j];
      isid[e] = id1[j];
      qi[e] = j < n_in ? qp->q[(int64_t)o * g->n_in + jidx(src[j], g->n_in)] : 0;
    }
  uint8_t *mask = out->spike_mask ? out->spike_mask : (uint8_t *)malloc(NL);
  uint8_t *ovf = out->overflowed ? out->overflowed : (uint8_t *)malloc(NL);
  run_layer_traced(a, isid, qi, qp->vth, n, L, qp->f_a, qp->f_V, qp->i_V, qp->round_mode,
                   qp->overflow_mode, mask, ovf, out->v_final, out->vmin, out->vmax,
                   out->v_steps);
  if (out->event_ms) /* trace.py:25-37 resolve_ms_fc: the column is the global event index */
    for (int32_t o = 0; o < n; ++o)
      for (int32_t j = 0; j < L; ++j)
        out->event_ms[(size_t)o * L + j] = j >= n_in ? (float)NAN : times[j];
  so_extract_output_events(mask, NULL, n, L, NULL, 1, L, times, E_len, g->max_out_spikes,
                           out->out_times, out->out_src, &out->n_real_out);
  out->spike_count = out->n_real_out;
  out->needed_queue = 0;
  reduce_layer(out, n, L, ovf);
  out->fits = out->n_real_out <= g->max_out_spikes && 0 <= g->max_extra_steps;
  if (!out->spike_mask) free(mask);
  if (!out->overflowed) free(ovf);
  free(dt);
  free(a1);
  free(id1);
  free(a);
  free(isid);
  free(qi);
  return 0;
}

/* ---- multi-threaded batch driver (CPU baseline only) ---- */
typedef struct {
  const so_layer_spec *layers;
  int32_t n_layers;
  const float *times;
  const int32_t *src, *n_real;
  int32_t B, E_len;
  int32_t *v_final_last, *spike_counts, *fits;
  atomic_int next;
  atomic_int err;
} batch_ctx;

static int32_t layer_neurons(const so_layer_spec *l) {
  if (l->kind == 1) return l->fc.n_out;
  const so_conv_geom *g = &l->conv;
  return g->oc * conv_h_out(g) * conv_w_out(g);
}

static void *batch_worker(void *arg) {
  batch_ctx *c = (batch_ctx *)arg;
  for (;;) {
    int b = atomic_fetch_add(&c->next, 1);
    if (b >= c->B) break;
    const float *t = c->times + (int64_t)b * c->E_len;
    const int32_t *s = c->src + (int64_t)b * c->E_len;
    int32_t E = c->E_len, nin = c->n_real[b];
    float *t_own = NULL;
    int32_t *s_own = NULL;
    int fits = 1;
    for (int32_t l = 0; l < c->n_layers; ++l) {
      const so_layer_spec *ls = &c->layers[l];
      int32_t n = layer_neurons(ls);
      int32_t M = ls->kind == 1 ? ls->fc.max_out_spikes : ls->conv.max_out_spikes;
      so_layer_out o;
      memset(&o, 0, sizeof(o));
      o.v_final = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
      o.vmin = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
      o.vmax = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
      o.out_times = (float *)malloc(sizeof(float) * (size_t)(M > 0 ? M : 1));
      o.out_src = (int32_t *)malloc(sizeof(int32_t) * (size_t)(M > 0 ? M : 1));
      int rc = ls->kind == 1 ? so_fc_forward(&ls->fc, &ls->qp, t, s, E, nin, &o)
                             : so_conv_forward(&ls->conv, &ls->qp, t, s, E, nin, &o);
      if (rc) atomic_store(&c->err, rc);
      fits = fits && o.fits;
      c->spike_counts[(int64_t)b * c->n_layers + l] = o.spike_count;
      if (l == c->n_layers - 1)
        memcpy(c->v_final_last + (int64_t)b * n, o.v_final, sizeof(int32_t) * (size_t)n);
      free(t_own);
      free(s_own);
      t_own = o.out_times;
      s_own = o.out_src;
      t = t_own;
      s = s_own;
      E = M;
      nin = o.n_real_out;
      free(o.v_final);
      free(o.vmin);
      free(o.vmax);
    }
    c->fits[b] = fits;
    free(t_own);
    free(s_own);
  }
  return NULL;
}

int so_network_batch(const so_layer_spec *layers, int32_t n_layers, const float *times,
                     const int32_t *src, const int32_t *n_real, int32_t B, int32_t E_len,
                     int32_t threads, int32_t *v_final_last, int32_t *spike_counts,
                     int32_t *fits) {
  batch_ctx c;
  c.layers = layers;
  c.n_layers = n_layers;
  c.times = times;
  c.src = src;
  c.n_real = n_real;
  c.B = B;
  c.E_len = E_len;
  c.v_final_last = v_final_last;
  c.spike_counts = spike_counts;
  c.fits = fits;
  atomic_init(&c.next, 0);
  atomic_init(&c.err, 0);
  if (threads < 1) threads = 1;
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
  for (int i = 0; i < threads; ++i) pthread_create(&th[i], NULL, batch_worker, &c);
  for (int i = 0; i < threads; ++i) pthread_join(th[i], NULL);
  free(th);
  return atomic_load(&c.err);
}

/* ================================================================ float chunked scan */

/* float/affine.py:20-24 combine(left, right): the map `right` applied after `left`. */
static inline void affine_combine(float la, float lb, float ra, float rb, float *oa, float *ob) {
  *oa = ra * la;
  *ob = ra * lb + rb;
}

/* lax.associative_scan's recursion (JAX, associative_scan._scan): combine neighbouring pairs,
 * scan the n/2 pair maps recursively (these are the prefixes ending at odd indices), then
 * combine each odd prefix with the following even-index map; element 0 is its own prefix.
 * work holds at least 4n floats. */
static void affine_scan_rec(const float *a, const float *b, int64_t n, float *oa, float *ob,
                            float *work) {
  if (n < 2) {
    if (n == 1) {
      oa[0] = a[0];
      ob[0] = b[0];
    }
    return;
  }
  const int64_t m = n / 2;
  float *ra = work, *rb = work + m, *sa = work + 2 * m, *sb = work + 3 * m, *next = work + 4 * m;
  for (int64_t i = 0; i < m; ++i)
    affine_combine(a[2 * i], b[2 * i], a[2 * i + 1], b[2 * i + 1], &ra[i], &rb[i]);
  affine_scan_rec(ra, rb, m, sa, sb, next);
  oa[0] = a[0];
  ob[0] = b[0];
  const int64_t n_even = (n % 2 == 0) ? m - 1 : m;
  for (int64_t i = 0; i < n_even; ++i)
    affine_combine(sa[i], sb[i], a[2 * i + 2], b[2 * i + 2], &oa[2 * i + 2], &ob[2 * i + 2]);
  for (int64_t i = 0; i < m; ++i) {
    oa[2 * i + 1] = sa[i];
    ob[2 * i + 1] = sb[i];
  }
}

int so_affine_scan(const float *a, const float *b, int64_t n, float *out_a, float *out_b) {
  if (n < 0) return -1;
  float *work = (float *)malloc(sizeof(float) * (size_t)(4 * n + 8));
  if (!work) return -2;
  affine_scan_rec(a, b, n, out_a, out_b, work);
  free(work);
  return 0;
}

typedef struct {
  int32_t *step, *j; /* the neuron's spikes: scan step and global event index */
  int32_t n, cap;
  int32_t step0_idx; /* spike_event_idx[neuron, 0] */
  uint8_t step0_spk; /* spike_mask[neuron, 0] */
  int32_t extra;     /* extra_steps_upper_bound - base_scan_steps for this neuron */
} fneuron_t;

typedef struct {
  const so_float_fc_geom *g;
  const float *w, *decay_base, *times, *gain;
  const int32_t *src;
  int32_t L, n_real, max_steps;
  so_float_out *out;
  fneuron_t *nr;
  atomic_int next, err;
} float_ctx;

static int push_spike(fneuron_t *r, int32_t step, int32_t j) {
  if (r->n == r->cap) {
    int32_t cap = r->cap ? 2 * r->cap : 64;
    int32_t *s = (int32_t *)realloc(r->step, sizeof(int32_t) * (size_t)cap);
    if (!s) return -2;
    r->step = s;
    int32_t *jj = (int32_t *)realloc(r->j, sizeof(int32_t) * (size_t)cap);
    if (!jj) return -2;
    r->j = jj;
    r->cap = cap;
  }
  r->step[r->n] = step;
  r->j[r->n] = j;
  ++r->n;
  return 0;
}

/* One neuron: fc_float_values (connectivity/fc.py:36-51) + float/scan.py:67-116 step loop +
 * affine.py:57-88 bound. */
static int float_neuron(float_ctx *c, int32_t i, float *a_pad, float *b_pad, float *ca, float *cb,
                        float *A, float *B, float *work) {
  const so_float_fc_geom *g = c->g;
  const int32_t L = c->L, C = g->chunk_size, Lp = L + C;
  const float base = c->decay_base[i], v_th = g->v_th;
  fneuron_t *r = &c->nr[i];
  /* build_fc_structure (fc.py:20-33): gap to the previous entry (the first against t=0), 0 on
   * pads; create_affine_maps (affine.py:27-31); mask_pad_events (affine.py:42-54);
   * _pad_queue (scan.py:19-25) appends chunk_size identity maps. */
  int32_t m_pos = 0;
  float sum_pos = 0.0f;
  for (int32_t j = 0; j < Lp; ++j) {
    float a = 1.0f, b = 0.0f;
    if (j < L && j < c->n_real) {
      const float prev = j == 0 ? 0.0f : c->times[j - 1];
      const float dt = c->times[j] - prev;
      a = powf(base, dt);
      b = c->w[(int64_t)i * g->n_in + jidx(c->src[j], g->n_in)];
      if (c->gain) b = b * c->gain[j];
    }
    a_pad[j] = a;
    b_pad[j] = b;
    if (j < L) { /* spike_step_upper_bound sums over the (n, L) maps, pads included as b = 0 */
      m_pos += b > 0.0f;
      sum_pos += b > 0.0f ? b : 0.0f;
    }
  }
  const float m_star = fminf((float)m_pos, floorf(sum_pos / v_th));
  const float steps_f = m_star + ceilf(((float)L - m_star) / (float)C);
  r->extra = f32_to_i32(steps_f) - (L + C - 1) / C;

  float v = 0.0f;
  int64_t ptr = 0;
  uint8_t *mask = c->out->spike_mask ? c->out->spike_mask + (int64_t)i * c->max_steps : NULL;
  int32_t *eidx = c->out->spike_event_idx ? c->out->spike_event_idx + (int64_t)i * c->max_steps
                                          : NULL;
  const int64_t id_from = L < c->n_real ? L : (c->n_real > 0 ? c->n_real : 0);
  float *vst = c->out->v_steps ? c->out->v_steps + (int64_t)i * c->max_steps : NULL;
  float *ems = c->out->event_ms ? c->out->event_ms + (int64_t)i * c->max_steps : NULL;
  for (int32_t step = 0; step < c->max_steps; ++step) {
    /* trace.py:25-37 resolve_ms_fc: the step's start pointer, idle from n_real on */
    if (ems) ems[step] = ptr >= c->n_real ? NAN : c->times[ptr < L - 1 ? ptr : L - 1];
    if (ptr >= id_from && !(v - v_th >= 0.0f)) {
      /* Every map from here on is the identity (1, 0), which composes to exactly (1, 0): each
       * remaining step leaves v unchanged, does not fire and consumes a whole chunk. */
      for (; step < c->max_steps; ++step) {
        const int32_t ev = (int32_t)(ptr + C < INT32_MAX ? ptr + C : INT32_MAX);
        if (ems) ems[step] = ptr >= c->n_real ? NAN : c->times[ptr < L - 1 ? ptr : L - 1];
        if (vst) vst[step] = v;
        if (mask) mask[step] = 0;
        if (eidx) eidx[step] = ev;
        if (step == 0) {
          r->step0_idx = ev;
          r->step0_spk = 0;
        }
        ptr += C;
      }
      break;
    }
    for (int32_t k = 0; k < C; ++k) { /* take_chunk: jnp.take(..., mode='clip') */
      int64_t idx = ptr + k;
      if (idx > Lp - 1) idx = Lp - 1;
      ca[k] = a_pad[idx];
      cb[k] = b_pad[idx];
    }
    affine_scan_rec(ca, cb, C, A, B, work);
    int32_t sidx = C; /* process_chunk (affine.py:99-126) */
    float v_spk = 0.0f;
    for (int32_t k = 0; k < C; ++k) {
      const float vs = A[k] * v + B[k];
      if (vs - v_th >= 0.0f) {
        sidx = k;
        v_spk = vs;
        break;
      }
    }
    const int spiked = sidx < C;
    v = spiked ? (1.0f - 1.0f) * v_spk : A[C - 1] * v + B[C - 1];
    const int32_t ev = (int32_t)(ptr + sidx);
    if (vst) vst[step] = v;
    if (mask) mask[step] = (uint8_t)spiked;
    if (eidx) eidx[step] = ev;
    if (step == 0) {
      r->step0_idx = ev;
      r->step0_spk = (uint8_t)spiked;
    }
    if (spiked && push_spike(r, step, ev)) return -2;
    ptr += spiked ? sidx + 1 : C;
  }
  c->out->v_final[i] = v;
  return 0;
}

static void *float_worker(void *arg) {
  float_ctx *c = (float_ctx *)arg;
  const int32_t C = c->g->chunk_size, Lp = c->L + C;
  float *a_pad = (float *)malloc(sizeof(float) * (size_t)Lp);
  float *b_pad = (float *)malloc(sizeof(float) * (size_t)Lp);
  float *buf = (float *)malloc(sizeof(float) * (size_t)(8 * C + 8));
  if (!a_pad || !b_pad || !buf) {
    atomic_store(&c->err, -2);
  } else {
    for (;;) {
      const int i = atomic_fetch_add(&c->next, 1);
      if (i >= c->g->n_out) break;
      if (float_neuron(c, i, a_pad, b_pad, buf, buf + C, buf + 2 * C, buf + 3 * C, buf + 4 * C))
        atomic_store(&c->err, -2);
    }
  }
  free(a_pad);
  free(b_pad);
  free(buf);
  return NULL;
}

typedef struct {
  int64_t key, pos;
} fkey_t;

static int fkey_cmp(const void *x, const void *y) {
  const fkey_t *a = (const fkey_t *)x, *b = (const fkey_t *)y;
  if (a->key != b->key) return a->key < b->key ? -1 : 1;
  return a->pos < b->pos ? -1 : (a->pos > b->pos);
}

int so_float_fc_forward(const so_float_fc_geom *g, const float *w, const float *decay_base,
                        const float *times, const int32_t *src, const float *gain, int32_t L,
                        int32_t n_real, int32_t threads, so_float_out *out) {
  if (!g || g->n_out < 1 || g->n_in < 1 || g->chunk_size < 1 || L < 1 || g->max_out_spikes < 0 ||
      g->max_extra_steps < 0)
    return -1;
  if ((int64_t)L + g->chunk_size > (1 << 30)) return -1;
  float_ctx c;
  memset(&c, 0, sizeof(c));
  c.g = g;
  c.w = w;
  c.decay_base = decay_base;
  c.times = times;
  c.gain = gain;
  c.src = src;
  c.L = L;
  c.n_real = n_real;
  c.max_steps = (L + g->chunk_size - 1) / g->chunk_size + g->max_extra_steps;
  c.out = out;
  c.nr = (fneuron_t *)calloc((size_t)g->n_out, sizeof(fneuron_t));
  if (!c.nr) return -2;
  atomic_init(&c.next, 0);
  atomic_init(&c.err, 0);
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  int started = 0;
  for (int t = 1; t < threads; ++t)
    if (pthread_create(&tid[started], NULL, float_worker, &c) == 0) ++started;
  float_worker(&c);
  for (int t = 0; t < started; ++t) pthread_join(tid[t], NULL);
  int rc = atomic_load(&c.err);

  /* layers/fc.py:96-100, stream.py:49-64 _select_spikes + :24-46 _pack_stream */
  int64_t total = 0;
  int32_t extra = (int32_t)0x80000000u;
  for (int32_t i = 0; i < g->n_out; ++i) {
    total += c.nr[i].n;
    if (c.nr[i].extra > extra) extra = c.nr[i].extra;
  }
  const int32_t M = g->max_out_spikes;
  fkey_t *keys = (fkey_t *)malloc(sizeof(fkey_t) * (size_t)(M > 0 ? M : 1));
  int32_t *nidx = (int32_t *)malloc(sizeof(int32_t) * (size_t)(M > 0 ? M : 1));
  int32_t *jdx = (int32_t *)malloc(sizeof(int32_t) * (size_t)(M > 0 ? M : 1));
  float *sraw = (float *)malloc(sizeof(float) * (size_t)(M > 0 ? M : 1));
  if (!keys || !nidx || !jdx || !sraw) rc = -2;
  if (!rc) {
    int32_t k = 0;
    for (int32_t i = 0; i < g->n_out && k < M; ++i)
      for (int32_t s = 0; s < c.nr[i].n && k < M; ++s, ++k) {
        nidx[k] = i;
        jdx[k] = c.nr[i].j[s];
        sraw[k] = 1.0f;
      }
    for (; k < M; ++k) { /* jnp.nonzero fill_value=0: neuron 0, step 0 */
      nidx[k] = 0;
      jdx[k] = c.nr[0].step0_idx;
      sraw[k] = c.nr[0].step0_spk ? 1.0f : 0.0f;
    }
    for (int32_t q = 0; q < M; ++q) {
      keys[q].key = q < total ? jdx[q] : L;
      keys[q].pos = q;
    }
    qsort(keys, (size_t)M, sizeof(fkey_t), fkey_cmp);
    for (int32_t q = 0; q < M; ++q) {
      const int64_t p = keys[q].pos;
      const int32_t jj = jdx[p] < L - 1 ? jdx[p] : L - 1;
      out->out_times[q] = p < total ? times[jj] : SO_PAD_TIME;
      out->out_src[q] = nidx[p];
      out->out_gain[q] = sraw[p];
    }
    out->n_real_out = (int32_t)total;
    out->extra_steps_needed = extra;
    out->fits = total <= M && extra <= g->max_extra_steps;
  }
  for (int32_t i = 0; i < g->n_out; ++i) {
    free(c.nr[i].step);
    free(c.nr[i].j);
  }
  free(c.nr);
  free(keys);
  free(nidx);
  free(jdx);
  free(sraw);
  return rc;
}

/* ================================================================ float conv layer */

/* float/scan.py:67-116: max_steps steps over one neuron's padded queue (Lp = L + C maps).  Per
 * step it records the spike flag, the queue column of the step's spike (pointer + spike_idx,
 * scan.py:114; pointer + C on a silent step), the potential after the step and the pointer at
 * the step's start (run_layer_traced's v_steps / pointer_steps, scan.py:118-119); any output
 * may be NULL.  Maps from column id_from on are identities.  Returns v_final. */
static float float_chunk_scan(const float *a_pad, const float *b_pad, int32_t L, int32_t C,
                              int64_t id_from, int32_t max_steps, float v_th, float *ca,
                              float *cb, float *A, float *B, float *work, uint8_t *mask,
                              int32_t *eidx, float *v_steps, int32_t *ptr_steps) {
  const int64_t Lp = (int64_t)L + C;
  float v = 0.0f;
  int64_t ptr = 0;
  for (int32_t step = 0; step < max_steps; ++step) {
    const int32_t p32 = (int32_t)(ptr < INT32_MAX ? ptr : INT32_MAX);
    if (ptr >= id_from && !(v - v_th >= 0.0f)) {
      /* identities compose to (1, 0): v stays, nothing fires, a whole chunk per step */
      if (mask) mask[step] = 0;
      if (eidx) eidx[step] = (int32_t)(ptr + C < INT32_MAX ? ptr + C : INT32_MAX);
      if (v_steps) v_steps[step] = v;
      if (ptr_steps) ptr_steps[step] = p32;
      ptr += C;
      continue;
    }
    for (int32_t k = 0; k < C; ++k) { /* take_chunk: jnp.take(..., mode='clip') */
      int64_t idx = ptr + k;
      if (idx > Lp - 1) idx = Lp - 1;
      ca[k] = a_pad[idx];
      cb[k] = b_pad[idx];
    }
    affine_scan_rec(ca, cb, C, A, B, work);
    int32_t sidx = C; /* process_chunk (affine.py:99-126) */
    float v_spk = 0.0f;
    for (int32_t k = 0; k < C; ++k) {
      const float vs = A[k] * v + B[k];
      if (vs - v_th >= 0.0f) {
        sidx = k;
        v_spk = vs;
        break;
      }
    }
    const int spiked = sidx < C;
    v = spiked ? (1.0f - 1.0f) * v_spk : A[C - 1] * v + B[C - 1];
    if (mask) mask[step] = (uint8_t)spiked;
    if (eidx) eidx[step] = (int32_t)(ptr + sidx);
    if (v_steps) v_steps[step] = v;
    if (ptr_steps) ptr_steps[step] = p32;
    ptr += spiked ? sidx + 1 : C;
  }
  return v;
}

int so_float_conv_forward(const so_float_conv_geom *fg, const float *w, float decay_base,
                          const float *times, const int32_t *src, const float *gain,
                          int32_t E_len, int32_t n_in, so_float_conv_out *out) {
  if (!fg || !out) return -1;
  const so_conv_geom *g = &fg->conv;
  const int32_t L = g->max_queue_len, C = fg->chunk_size, K = g->k;
  if (C < 1 || L < 1 || E_len < 1 || g->max_extra_steps < 0 || g->max_out_spikes < 0)
    return -1;
  const int32_t h_out = conv_h_out(g), w_out = conv_w_out(g), n_sp = h_out * w_out;
  const int64_t n = (int64_t)g->oc * n_sp;
  const int32_t max_steps = (L + C - 1) / C + g->max_extra_steps;
  const int64_t nL = (int64_t)n_sp * L;
  int32_t *l2g = (int32_t *)malloc(sizeof(int32_t) * (size_t)nL * 4);
  int32_t *n_real = (int32_t *)malloc(sizeof(int32_t) * (size_t)n_sp);
  float *dt = (float *)malloc(sizeof(float) * (size_t)nL * 2);
  uint8_t *mask = out->spike_mask ? out->spike_mask
                                  : (uint8_t *)malloc((size_t)(n * max_steps));
  int32_t *eidx = out->spike_event_idx
                      ? out->spike_event_idx
                      : (int32_t *)malloc(sizeof(int32_t) * (size_t)(n * max_steps));
  int32_t *ptr_steps = out->event_ms ? (int32_t *)malloc(sizeof(int32_t) * (size_t)(n * max_steps))
                                     : NULL;
  const int32_t Lp = L + C;
  float *a_pad = (float *)malloc(sizeof(float) * (size_t)Lp * 2);
  float *buf = (float *)malloc(sizeof(float) * (size_t)(8 * C + 8));
  int rc = 0;
  if (!l2g || !n_real || !dt || !mask || !eidx || (out->event_ms && !ptr_steps) || !a_pad || !buf) {
    rc = -2;
    goto done;
  }
  {
    int32_t *tc = l2g + nL, *tky = l2g + 2 * nL, *tkx = l2g + 3 * nL;
    float *a_pos = dt + nL;
    float *b_pad = a_pad + Lp;
    rc = so_conv_structure(g, times, src, E_len, n_in, l2g, n_real, dt, tc, tky, tkx);
    if (rc) goto done;
    /* conv_float_values (connectivity/conv.py:187-206): a per position, tiled over channels */
    for (int64_t e = 0; e < nL; ++e) a_pos[e] = powf(decay_base, dt[e]);
    int32_t nq_max = 0, extra = (int32_t)0x80000000u;
    for (int32_t pos = 0; pos < n_sp; ++pos)
      if (n_real[pos] > nq_max) nq_max = n_real[pos];
    for (int64_t i = 0; i < n; ++i) {
      const int32_t oc = (int32_t)(i / n_sp), pos = (int32_t)(i % n_sp);
      const int32_t nr = n_real[pos];
      int32_t m_pos = 0;
      float sum_pos = 0.0f;
      for (int32_t col = 0; col < Lp; ++col) {
        float a = 1.0f, b = 0.0f;
        if (col < L) {
          const int64_t e = (int64_t)pos * L + col;
          a = a_pos[e];
          if (col < nr) { /* _real_tap_mask; weight gather with JAX clamping */
            const int64_t c = jidx(tc[e], g->ic);
            b = w[(((int64_t)oc * g->ic + c) * K + tky[e]) * K + tkx[e]];
            if (gain) {
              const int32_t ej = l2g[e] < n_in - 1 ? l2g[e] : n_in - 1;
              b = b * gain[jidx(ej, E_len)];
            }
          }
          m_pos += b > 0.0f; /* spike_step_upper_bound over the (n, L) b */
          sum_pos += b > 0.0f ? b : 0.0f;
        }
        a_pad[col] = a;
        b_pad[col] = b;
      }
      const float m_star = fminf((float)m_pos, floorf(sum_pos / fg->v_th));
      const float steps_f = m_star + ceilf(((float)L - m_star) / (float)C);
      const int32_t ex = f32_to_i32(steps_f) - (L + C - 1) / C;
      if (ex > extra) extra = ex;
      /* from the column after the catch-up column on, every map is the identity */
      const int64_t id_from = nr < L ? nr + 1 : L;
      const int64_t row = i * max_steps;
      out->v_final[i] = float_chunk_scan(
          a_pad, b_pad, L, C, id_from, max_steps, fg->v_th, buf, buf + C, buf + 2 * C,
          buf + 3 * C, buf + 4 * C, mask + row, eidx + row,
          out->v_steps ? out->v_steps + row : NULL, ptr_steps ? ptr_steps + row : NULL);
      if (out->event_ms) /* trace.py:40-55 resolve_ms_conv */
        for (int32_t s = 0; s < max_steps; ++s) {
          const int32_t p = ptr_steps[row + s];
          if (p >= nr) {
            out->event_ms[row + s] = NAN;
          } else {
            const int32_t col = p < L - 1 ? p : L - 1;
            const int32_t gj = l2g[(int64_t)pos * L + col];
            out->event_ms[row + s] = times[gj < E_len - 1 ? gj : E_len - 1];
          }
        }
    }
    /* layers/conv.py:133-141: output stream and needs */
    const int32_t M = g->max_out_spikes;
    int32_t nr_out = 0;
    so_extract_output_events(mask, eidx, (int32_t)n, max_steps, l2g, n_sp, L, times, E_len, M,
                             out->out_times, out->out_src, &nr_out);
    for (int32_t q = 0; q < M; ++q) /* s_spike: 1 on a fire; the fill entry is (neuron 0, step 0) */
      out->out_gain[q] = q < nr_out ? 1.0f : (mask[0] ? 1.0f : 0.0f);
    out->n_real_out = nr_out;
    out->needed_queue = nq_max + 1;
    out->extra_steps_needed = extra;
    out->fits = nq_max + 1 <= L && nr_out <= M && extra <= g->max_extra_steps;
  }
done:
  if (!out->spike_mask) free(mask);
  if (!out->spike_event_idx) free(eidx);
  free(ptr_steps);
  free(l2g);
  free(n_real);
  free(dt);
  free(a_pad);
  free(buf);
  return rc;
}

/* ---------------------------------------------------------------- float64 yardstick */

int so_float_seq64(int32_t n_in, int32_t n_out, const float *w, const float *decay_base,
                   const float *times, const int32_t *src, const float *gain, int32_t E_len,
                   int32_t n_real, int32_t chunk_size, int32_t max_extra_steps, double v_th,
                   double near, double *v_final, int32_t *first_near) {
  if (n_in < 1 || n_out < 1 || E_len < 0 || chunk_size < 1) return 1;
  const int32_t n_eff = n_real < 0 ? 0 : (n_real > E_len ? E_len : n_real);
  const int64_t max_steps = (E_len + chunk_size - 1) / chunk_size + (int64_t)max_extra_steps;
  const double band = near * fabs(v_th);
  for (int32_t o = 0; o < n_out; ++o) {
    double v = 0.0;
    int64_t phase = 0, steps = 0;
    int run = max_steps > 0;
    float tprev = 0.0f;
    int32_t fn = E_len;
    const double base = (double)decay_base[o];
    for (int32_t j = 0; j < n_eff && run; ++j) {
      const float t = times[j];
      const double dt = (double)(float)(t - tprev);
      tprev = t;
      int32_t s = src[j];
      if (s < 0) s += n_in;
      if (s < 0) s = 0;
      if (s >= n_in) s = n_in - 1;
      const double b = (double)w[(int64_t)o * n_in + s] * (gain ? (double)gain[j] : 1.0);
      v = pow(base, dt) * v + b;
      if (fn == E_len && fabs(v - v_th) < band) fn = j;
      const int spike = v >= v_th;
      if (spike) v = 0.0;
      phase += 1;
      if (spike || phase == chunk_size) {
        steps += 1;
        phase = 0;
      }
      run = steps < max_steps;
    }
    v_final[o] = v;
    first_near[o] = fn;
  }
  return 0;
}
