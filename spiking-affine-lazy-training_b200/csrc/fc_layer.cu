// Integer FC layer for B200 (sm_100a).
//
// Replaces FCLayer.forward with QuantBackend (salt_core/layers/fc.py:385-402): every output
// neuron scans the whole input stream (connectivity/fc.py:20-33 — Δt against the previous
// entry, the first against t=0, pads masked to Δt=0 and weight 0), applying
// quant/scan.py:22-52 per entry; spikes leave as per-event neuron bitmasks and are compacted
// into the next EventStream in (event, neuron) order (stream.py:24-81).
//
// fc_scan: one warp per (sample, group of 32 output neurons); lane = neuron.  Events are read
// 32 at a time (one coalesced load per lane) and broadcast with shuffles; the weight codes of
// the 32 events are fetched before the dependent recurrence so their latency overlaps.
// Pad entries are identity steps that can only fire when v_th_int <= 0, so they are walked
// only in that case (tail mode).
#include "salt_layers.cuh"

namespace salt {

// LPU lanes (one per output neuron) form a group that runs one (sample, 32-neuron group) unit;
// LPU < 32 packs 32 / LPU samples into a warp when the layer has at most LPU neurons (G == 1),
// as the membrane readout layers do.
template <bool FIRES, bool SAT, int LPU>
__global__ void __launch_bounds__(kFcThreads) fc_scan(FCLaunch P) {
  constexpr int SPW = 32 / LPU;
  constexpr uint32_t kAll = 0xffffffffu;
  __shared__ int32_t lut_s[kLutSmemMax];
  const bool lut_smem = P.qc.lut_len <= kLutSmemMax;
  if (lut_smem)
    for (int i = threadIdx.x; i < P.qc.lut_len; i += blockDim.x) lut_s[i] = P.lut[i];
  __syncthreads();
  const int32_t* lut = lut_smem ? lut_s : P.lut;
  const int lane = threadIdx.x & 31, gi = lane / LPU, gl = lane % LPU;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t n_units = (int64_t)P.batch * P.G;
  if (gw * SPW >= n_units) return;  // the whole warp is past the last unit
  const int64_t unit = gw * SPW + gi;
  const bool unit_ok = unit < n_units;
  const int b = unit_ok ? (int)(unit / P.G) : 0, g = unit_ok ? (int)(unit % P.G) : 0;
  const int o = g * LPU + gl;
  const bool active = unit_ok && o < P.n_out;
  const int32_t n_in = unit_ok ? P.in_nreal[b] : 0;
  const int32_t n_eff = unit_ok ? P.n_eff(b) : 0;
  const int32_t nproc = !unit_ok ? 0 : (P.tail_mode ? P.in.capacity : n_eff);
  // lanes past n_out never fire (their register stays 0); registers stay below INT32_MAX
  const int32_t vth = (FIRES && active) ? P.vth[o] : INT32_MAX;
  const StepConsts sc(P.qc);
  uint32_t* sw_b = FIRES ? P.sw + (int64_t)b * P.sw_stride : nullptr;
  int32_t* chunk_b = FIRES ? P.chunk_spikes + (int64_t)b * P.n_spk_chunks : nullptr;
  const int32_t nmax = __reduce_max_sync(kAll, nproc);

  int32_t V = 0, vmin = 0, vmax = 0, nspk = 0;
  float tprev = 0.0f;
  for (int32_t base = 0; base < nmax; base += LPU) {
    // Lane-parallel preparation of LPU events: time, source, Δt against the previous entry
    // (connectivity/fc.py:26-29: the first against t=0, pads masked to 0) and decay code.
    const int32_t jl = base + gl;
    float t_l = 0.0f;
    int32_t s_l = 0;
    if (jl < nproc) {
      t_l = P.in.time(b, jl, n_eff);
      s_l = P.in.source(b, jl, n_eff);
    }
    float t_prev_l = __shfl_up_sync(kAll, t_l, 1, LPU);
    if (gl == 0) t_prev_l = tprev;
    const bool real_l = jl < n_in;
    const int32_t dt_l = real_l ? dt_from_times(t_l, t_prev_l) : 0;
    const int32_t a_l = dt_l == 0 ? sc.ident_a : decay_code(dt_l, lut, P.qc.lut_len);
    const int cnt = min(LPU, nproc - base);  // this group's events in the batch (may be <= 0)
    const float t_last = __shfl_sync(kAll, t_l, cnt > 0 ? cnt - 1 : 0, LPU);
    if (cnt > 0) tprev = t_last;
    int32_t qv[LPU];
#pragma unroll
    for (int e = 0; e < LPU; ++e) {
      const int32_t s = __shfl_sync(kAll, s_l, e, LPU);
      const bool real = (base + e) < n_in && e < cnt;  // fc.py:29 is_real = j < n_real
      qv[e] = (real && active) ? __ldg(&P.qT[jax_index(s, P.n_in) * P.n_out + o]) : 0;
    }
    const int cntw = min(LPU, nmax - base);  // warp-uniform batch length
#pragma unroll
    for (int e = 0; e < LPU; ++e) {
      if (e < cntw) {
        const int32_t a = __shfl_sync(kAll, a_l, e, LPU);
        bool spike = false;
        if (e < cnt) {
          int32_t u;
          const int32_t w = sc.step<SAT>(V, a, qv[e], u);
          spike = FIRES && w >= vth;
          V = spike ? 0 : w;
          // inactive lanes see q = 0 from V = 0, so u = 0 leaves the range untouched; overflow
          // is read off the unfitted range at the end of the layer (layer_finish)
          vmin = min(vmin, u);
          vmax = max(vmax, u);
          nspk += spike;
        }
        if (FIRES) {
          const uint32_t bal = __ballot_sync(kAll, spike);
          const uint32_t bits = LPU == 32 ? bal : (bal >> (gi * LPU)) & ((1u << LPU) - 1u);
          if (gl == 0 && e < cnt) {
            const int32_t j = base + e;
            sw_b[(int64_t)j * P.G + g] = bits;
            if (bits) atomicAdd(&chunk_b[j >> kSpkChunkShift], __popc(bits));
          }
        }
      }
    }
  }
  if (active) P.v_final[(int64_t)b * P.n_out + o] = V;
  if (FIRES && active) P.n_spk[(int64_t)b * P.n_out + o] = nspk;
  // per-group reductions (lanes of other groups belong to other samples)
#pragma unroll
  for (int off = LPU / 2; off > 0; off >>= 1) {
    vmin = min(vmin, __shfl_xor_sync(kAll, vmin, off, LPU));
    vmax = max(vmax, __shfl_xor_sync(kAll, vmax, off, LPU));
    nspk += __shfl_xor_sync(kAll, nspk, off, LPU);
  }
  if (gl == 0 && unit_ok) {
    atomicMin(&P.vmin[b], vmin);
    atomicMax(&P.vmax[b], vmax);
    if (nspk) atomicAdd(&P.s_total[b], nspk);
  }
}


// Emits sample b's spikes in (event, neuron) order; block x walks the sample's 256-event
// chunks x, x + gridDim.x, ... (chunk offsets come from the scanned per-chunk counts).
__global__ void __launch_bounds__(kCompactThreads)
fc_compact(FCLaunch P, salt_stream_out out) {
  __shared__ int32_t s_scan[kScanSmem];
  const int b = blockIdx.y, tid = threadIdx.x;
  if (P.s_total[b] > P.M) return;
  const int32_t n_eff = P.n_eff(b);
  const int32_t nproc = P.tail_mode ? P.in.capacity : n_eff;
  for (int32_t c = blockIdx.x; c * kSpkChunk < nproc; c += gridDim.x) {
    const int32_t j = c * kSpkChunk + tid;
    const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * P.G;
    int32_t cnt = 0;
    if (j < nproc)
      for (int g = 0; g < P.G; ++g) cnt += __popc(sw_j[g]);
    int32_t total;
    const int32_t off = block_exclusive_scan(cnt, s_scan, total);
    if (cnt == 0) continue;
    int32_t k = P.chunk_off[(int64_t)b * P.n_spk_chunks + c] + off;
    const float t = P.in.time(b, j, n_eff);
    for (int g = 0; g < P.G; ++g) {
      uint32_t wd = sw_j[g];
      while (wd) {
        const int bit = __ffs(wd) - 1;
        wd &= wd - 1u;
        out.times[(int64_t)b * P.M + k] = t;
        out.src[(int64_t)b * P.M + k] = g * 32 + bit;
        ++k;
      }
    }
  }
}

// Samples with more than max_out spikes keep the first M in neuron-major order (stream.py:60):
// every spike of neurons < n*, and the first r of neuron n* (by event index).
__global__ void __launch_bounds__(kCompactThreads)
fc_truncated(FCLaunch P, salt_stream_out out) {
  __shared__ int32_t s_scan[kScanSmem];
  __shared__ int32_t s_cut[4];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int32_t S = P.s_total[b], M = P.M;
  if (S <= M || M <= 0) return;
  const int32_t n_eff = P.n_eff(b);
  const int32_t nproc = P.tail_mode ? P.in.capacity : n_eff;
  if (tid == 0) {
    int32_t cum = 0, nst = P.n_out - 1;
    for (int o = 0; o < P.n_out; ++o) {
      const int32_t c = P.n_spk[(int64_t)b * P.n_out + o];
      if (cum + c >= M) {
        nst = o;
        break;
      }
      cum += c;
    }
    s_cut[0] = nst;
    s_cut[1] = M - cum;
    s_cut[2] = 0x7fffffff;
  }
  __syncthreads();
  const int nst = s_cut[0], gq = nst >> 5, bq = nst & 31;
  int32_t seen = 0;
  for (int32_t j0 = 0; j0 < nproc; j0 += blockDim.x) {
    const int32_t j = j0 + tid;
    const int32_t hit =
        j < nproc ? (int32_t)((P.sw[(int64_t)b * P.sw_stride + (int64_t)j * P.G + gq] >> bq) & 1u)
                  : 0;
    int32_t total;
    const int32_t off = block_exclusive_scan(hit, s_scan, total);
    if (hit && seen + off + 1 == s_cut[1]) s_cut[2] = j;
    seen += total;
    __syncthreads();
    if (s_cut[2] != 0x7fffffff) break;
  }
  __syncthreads();
  const int32_t j_cut = s_cut[2];
  int32_t written = 0;
  for (int32_t j0 = 0; j0 < nproc; j0 += blockDim.x) {
    const int32_t j = j0 + tid;
    const uint32_t* sw_j = P.sw + (int64_t)b * P.sw_stride + (int64_t)j * P.G;
    int32_t cnt = 0;
    if (j < nproc)
      for (int g = 0; g < P.G; ++g) {
        uint32_t wd = sw_j[g];
        while (wd) {
          const int o = g * 32 + __ffs(wd) - 1;
          wd &= wd - 1u;
          cnt += (o < nst) || (o == nst && j <= j_cut);
        }
      }
    int32_t total;
    const int32_t off = block_exclusive_scan(cnt, s_scan, total);
    if (cnt) {
      const float t = P.in.time(b, j, n_eff);
      int32_t k = written + off;
      for (int g = 0; g < P.G; ++g) {
        uint32_t wd = sw_j[g];
        while (wd) {
          const int o = g * 32 + __ffs(wd) - 1;
          wd &= wd - 1u;
          if ((o < nst) || (o == nst && j <= j_cut)) {
            out.times[(int64_t)b * M + k] = t;
            out.src[(int64_t)b * M + k] = o;
            ++k;
          }
        }
      }
    }
    written += total;
  }
}

template <int LPU>
static void* fc_scan_for(bool fires, bool saturate) {
  if (saturate) return fires ? (void*)fc_scan<true, true, LPU> : (void*)fc_scan<false, true, LPU>;
  return fires ? (void*)fc_scan<true, false, LPU> : (void*)fc_scan<false, false, LPU>;
}

void* fc_scan_kernel(bool fires, bool saturate, int lpu) {
  if (lpu == 8) return fc_scan_for<8>(fires, saturate);
  if (lpu == 16) return fc_scan_for<16>(fires, saturate);
  return fc_scan_for<32>(fires, saturate);
}

}  // namespace salt
