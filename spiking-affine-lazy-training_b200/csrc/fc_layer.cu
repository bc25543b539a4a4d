// Integer FC layer for B200 (sm_100a).
//
// Replaces FCLayer.forward with QuantBackend (salt_core/layers/fc.py:84-101): every output
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

template <int WT> struct CodeType { using T = int32_t; };
template <> struct CodeType<1> { using T = int8_t; };
template <> struct CodeType<2> { using T = int16_t; };

// Shared-memory layout of fc_scan: decay table (when short enough), then the per-warp event
// records, then (WT > 0) the block's neuron group's weight codes, (n_in, q_cols) followed by a
// zero row that masked entries point at.
__host__ __device__ inline int fc_lut_words(int32_t lut_len) {
  return lut_len <= kLutSmemMax ? ((lut_len + 3) & ~3) : 0;
}
__host__ __device__ inline int fc_ring(int wt) { return wt ? kFcRing : 1; }

// Columns of the staged weight table: a layer of one neuron group stages its whole (n_in, n_out)
// table; otherwise each block stages the LPU columns of its own group.
__host__ __device__ inline int32_t fc_q_cols(int32_t n_out, int lpu) {
  return n_out <= lpu ? n_out : lpu;
}

size_t fc_scan_q_bytes(int32_t n_in, int32_t n_out, int wt, int lpu) {
  // + one zero row of lpu entries: masked entries and lanes past n_out read it
  return wt ? (((size_t)n_in * fc_q_cols(n_out, lpu) + lpu) * wt + 15) & ~(size_t)15 : 0;
}

size_t fc_scan_smem(int32_t n_in, int32_t n_out, int32_t lut_len, int wt, int lpu) {
  const size_t ev = (size_t)(kFcThreads / 32) * (32 / lpu) * lpu * fc_ring(wt) * sizeof(int2);
  const size_t q = fc_scan_q_bytes(n_in, n_out, wt, lpu);
  return (size_t)fc_lut_words(lut_len) * 4 + ev + q;
}

// LPU lanes (one per output neuron) form a group that runs one (sample, 32-neuron group) unit;
// LPU < 32 packs 32 / LPU samples into a warp when the layer has at most LPU neurons (G == 1),
// as the membrane readout layers do.
//
// The recurrence of one unit is a dependent chain of a few integer operations per event, so the
// kernel is latency-bound; everything else is taken off the chain.  Events arrive in
// super-batches of R * LPU (R events per lane, coalesced), and the next super-batch's loads are
// in flight while the current one runs.  Each event's decay code and weight-row offset are
// computed lane-parallel and parked as one int2 per event in shared memory, which every lane of
// the group then reads with one broadcast load per step.  With WT > 0 the weight codes sit in
// shared memory as WT-byte integers with a zero row that masked entries (pads, events past the
// group's end) point at, so a step needs no predicate: past the end it is the identity.
template <bool FIRES, bool SAT, int LPU, int WT, int FORM>
__global__ void __launch_bounds__(kFcThreads) fc_scan(FCLaunch P) {
  using QT = typename CodeType<WT>::T;
  constexpr int SPW = 32 / LPU;
  constexpr int R = WT ? kFcRing : 1;
  constexpr int SB = R * LPU;
  constexpr uint32_t kAll = 0xffffffffu;
  extern __shared__ __align__(16) unsigned char fc_smem[];
  const int lut_words = fc_lut_words(P.qc.lut_len);
  int32_t* lut_s = reinterpret_cast<int32_t*>(fc_smem);
  int2* ev_all = reinterpret_cast<int2*>(fc_smem + (size_t)lut_words * 4);
  QT* q_s = reinterpret_cast<QT*>(ev_all + (kFcThreads / 32) * SPW * SB);
  const int g = blockIdx.y;  // the block's neuron group: neurons [g * LPU, g * LPU + LPU)
  const int32_t qcols = fc_q_cols(P.n_out, LPU);
  const int32_t zero_row = P.n_in * qcols;
  if (lut_words)
    for (int i = threadIdx.x; i < P.qc.lut_len; i += blockDim.x) lut_s[i] = P.lut[i];
  if (WT) {
    // kStageLoads loads per thread are issued before any is stored, so the staging costs a few
    // global latencies instead of one per code (a block of a narrow layer stages its whole table
    // and the sample chains start only after it)
    for (int32_t i0 = threadIdx.x; i0 < zero_row; i0 += blockDim.x * kStageLoads) {
      int32_t v[kStageLoads];
#pragma unroll
      for (int u = 0; u < kStageLoads; ++u) {
        const int32_t i = i0 + u * (int32_t)blockDim.x;
        v[u] = 0;
        if (i < zero_row) {
          if (P.G == 1) {  // the whole table, as laid out in global memory
            v[u] = __ldg(&P.qT[i]);
          } else {         // this group's LPU columns
            const int32_t row = i / LPU, col = g * LPU + (i - row * LPU);
            if (col < P.n_out) v[u] = __ldg(&P.qT[(int64_t)row * P.n_out + col]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kStageLoads; ++u) {
        const int32_t i = i0 + u * (int32_t)blockDim.x;
        if (i < zero_row) q_s[i] = (QT)v[u];
      }
    }
    for (int32_t i = threadIdx.x; i < LPU; i += blockDim.x) q_s[zero_row + i] = 0;
  }
  __syncthreads();
  const int32_t* lut = lut_words ? lut_s : P.lut;
  const int lane = threadIdx.x & 31, gi = lane / LPU, gl = lane % LPU;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw * SPW >= P.batch) return;  // the whole warp is past the last sample
  int2* ev_s = ev_all + ((threadIdx.x >> 5) * SPW + gi) * SB;
  const int64_t bs = gw * SPW + gi;  // sample slot
  const bool unit_ok = bs < P.batch;
  // samples in heaviest-first order: a warp's samples have similar lengths, and the longest
  // chains start first
  const int b = !unit_ok ? 0 : (P.order ? P.order[bs] : (int)bs);
  const int o = g * LPU + gl;
  const bool active = unit_ok && o < P.n_out;
  const int32_t n_in = unit_ok ? P.in_nreal[b] : 0;
  const int32_t n_eff = unit_ok ? P.n_eff(b) : 0;
  const int32_t nproc = !unit_ok ? 0 : (P.tail_mode ? P.in.capacity : n_eff);
  // lanes past n_out never fire (their register stays 0 or runs column 0 without firing);
  // registers stay below INT32_MAX
  const int32_t vth = (FIRES && active) ? P.vth[o] : INT32_MAX;
  const StepConsts sc(P.qc);
  uint32_t* sw_b = FIRES ? P.sw + (int64_t)b * P.sw_stride : nullptr;
  int32_t* chunk_b = FIRES ? P.chunk_spikes + (int64_t)b * P.n_spk_chunks : nullptr;
  const int32_t nmax = __reduce_max_sync(kAll, nproc);

  // the input stream is read two super-batches ahead: a super-batch's chain is shorter than a
  // global load's latency at the occupancy of a narrow layer (one warp per scheduler)
  float tn[R], tn2[R];
  int32_t sn[R], sn2[R];
  auto load = [&](int32_t base, float (&t)[R], int32_t (&sv)[R]) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int32_t j = base + r * LPU + gl;
      t[r] = 0.0f;
      sv[r] = 0;
      if (j < nproc) {
        t[r] = P.in.time(b, j, n_eff);
        sv[r] = P.in.source(b, j, n_eff);
      }
    }
  };
  load(0, tn, sn);
  load(SB, tn2, sn2);
  int32_t V = 0, vmin = 0, vmax = 0, nspk = 0;
  float tcarry = 0.0f;
  for (int32_t base = 0; base < nmax; base += SB) {
    float tc[R];
    int32_t scur[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      tc[r] = tn[r];
      scur[r] = sn[r];
      tn[r] = tn2[r];
      sn[r] = sn2[r];
    }
    if (base + 2 * SB < nmax) load(base + 2 * SB, tn2, sn2);  // in flight for two super-batches
    // lane-parallel: Δt against the previous entry (connectivity/fc.py:26-29: the first
    // against t = 0, pads masked to Δt = 0 and weight 0), decay code and weight-row offset
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int32_t j = base + r * LPU + gl;
      float tp = __shfl_up_sync(kAll, tc[r], 1, LPU);
      // the group's first lane continues from the previous row of events (or super-batch)
      const float row_prev = r ? __shfl_sync(kAll, tc[r > 0 ? r - 1 : 0], LPU - 1, LPU) : tcarry;
      if (gl == 0) tp = row_prev;
      const bool real = j < n_in && j < nproc;
      const int32_t dt = real ? dt_from_times(tc[r], tp) : 0;
      const int32_t a = dt == 0 ? sc.ident_a : decay_code(dt, lut, P.qc.lut_len);
      int32_t qo;  // row offset of the event's weights (staged table, or the global codes)
      if (WT) qo = real ? (int32_t)jax_index(scur[r], P.n_in) * qcols : zero_row;
      else qo = real ? (int32_t)jax_index(scur[r], P.n_in) * P.n_out + g * LPU : -1;
      ev_s[r * LPU + gl] = make_int2(a, qo);
    }
    tcarry = __shfl_sync(kAll, tc[R - 1], LPU - 1, LPU);
    __syncwarp();
    const int32_t cnt = nproc - base;  // this group's events in the super-batch (may be <= 0)
    const int32_t cntw = min(SB, nmax - base);
    uint32_t mybits[R];
    int32_t sb_spk = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) mybits[r] = 0;
    // lanes past n_out read the row's tail (or the zero row's padding); their results are
    // dropped
    auto load_q = [&](int32_t row) -> int32_t {
      if (WT) return (int32_t)q_s[row + gl];
      return (row >= 0 && active) ? __ldg(&P.qT[row + gl]) : 0;
    };
    auto step_with = [&](int e, int32_t a, int32_t qv) {
      int32_t u;
      const int32_t w = sc.step<SAT, FORM != kStepSplit, FORM != kStepWideNoFit>(V, a, qv, u);
      vmin = min(vmin, u);
      vmax = max(vmax, u);
      if (FIRES) {
        const bool spike = w >= vth;
        V = spike ? 0 : w;
        nspk += spike;
        const uint32_t bal = __ballot_sync(kAll, spike);
        const uint32_t bits = LPU == 32 ? bal : (bal >> (gi * LPU)) & ((1u << (LPU & 31)) - 1u);
        if (gl == (e % LPU)) mybits[e / LPU] = bits;
        sb_spk += __popc(bits);
      } else {
        V = w;
      }
    };
    if (cntw == SB) {
      // blocks of kFcStepBlock steps: a block's (decay code, weight row) pairs and weight codes
      // are loaded together ahead of its dependent register chain, so the shared-memory
      // latencies overlap one another and the previous block's chain
#pragma unroll
      for (int e0 = 0; e0 < SB; e0 += kFcStepBlock) {
        int2 evb[kFcStepBlock];
        int32_t qb[kFcStepBlock];
#pragma unroll
        for (int k = 0; k < kFcStepBlock; ++k) evb[k] = ev_s[e0 + k];
#pragma unroll
        for (int k = 0; k < kFcStepBlock; ++k) qb[k] = load_q(evb[k].y);
#pragma unroll
        for (int k = 0; k < kFcStepBlock; ++k) step_with(e0 + k, evb[k].x, qb[k]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < SB; ++e)
        if (e < cntw) {
          const int2 ev = ev_s[e];
          step_with(e, ev.x, load_q(ev.y));
        }
    }
    if (FIRES) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int32_t j = base + r * LPU + gl;
        if (r * LPU + gl < cnt && unit_ok) sw_b[(int64_t)j * P.G + g] = mybits[r];
      }
      // a super-batch lies inside one spike-count chunk (SB divides kSpkChunk)
      if (gl == 0 && sb_spk && unit_ok) atomicAdd(&chunk_b[base >> kSpkChunkShift], sb_spk);
    }
    __syncwarp();
  }
  // pad columns the scan skipped are identity steps whose unfitted value is the register
  // (quant/scan.py:40-42); steps past a group's end above were such identity steps too
  if (!P.tail_mode && n_eff < P.in.capacity) {
    vmin = min(vmin, V);
    vmax = max(vmax, V);
  }
  if (!active) vmin = vmax = nspk = 0;
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

template <int LPU, int WT, int FORM>
static void* fc_scan_for(bool fires, bool saturate) {
  if (FORM == kStepWideNoFit)  // the overflow mode does not matter
    return fires ? (void*)fc_scan<true, false, LPU, WT, FORM>
                 : (void*)fc_scan<false, false, LPU, WT, FORM>;
  if (saturate)
    return fires ? (void*)fc_scan<true, true, LPU, WT, FORM>
                 : (void*)fc_scan<false, true, LPU, WT, FORM>;
  return fires ? (void*)fc_scan<true, false, LPU, WT, FORM>
               : (void*)fc_scan<false, false, LPU, WT, FORM>;
}

template <int WT, int FORM>
static void* fc_scan_lpu(bool fires, bool saturate, int lpu) {
  if (lpu == 8) return fc_scan_for<8, WT, FORM>(fires, saturate);
  if (lpu == 16) return fc_scan_for<16, WT, FORM>(fires, saturate);
  return fc_scan_for<32, WT, FORM>(fires, saturate);
}

template <int FORM>
static void* fc_scan_wt(bool fires, bool saturate, int lpu, int wt) {
  switch (wt) {
    case 1: return fc_scan_lpu<1, FORM>(fires, saturate, lpu);
    case 2: return fc_scan_lpu<2, FORM>(fires, saturate, lpu);
    case 4: return fc_scan_lpu<4, FORM>(fires, saturate, lpu);
    default: return fc_scan_lpu<0, FORM>(fires, saturate, lpu);
  }
}

void* fc_scan_kernel(bool fires, bool saturate, int lpu, int wt, int form) {
  if (form == kStepWideNoFit) return fc_scan_wt<kStepWideNoFit>(fires, saturate, lpu, wt);
  return form == kStepWide ? fc_scan_wt<kStepWide>(fires, saturate, lpu, wt)
                           : fc_scan_wt<kStepSplit>(fires, saturate, lpu, wt);
}

}  // namespace salt
