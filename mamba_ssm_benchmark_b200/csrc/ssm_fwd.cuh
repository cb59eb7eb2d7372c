// ssm_fwd.cuh — forward selective scan on sm_100a.
//
// Replaces the reference's forward GPU path, kernels/triton_scan.py:27-74 (_fwd_kernel) and
// :253-286 (_launch_fwd, TritonSelectiveScanFn.forward); the math is models/scan.py:39-55
// (discretize) and :70-76 (the recurrence h_t = a_t h_{t-1} + b_t), y_t = <C_t, h_t>.
//
// One warp (= one CTA) owns a (batch, CPW-channel slice, time segment) and walks the segment
// in 16-step tiles; its lane 0 streams boxes of KB tiles (KB = 2 or 4) through a 2-stage TMA
// ring: u, delta, z (16 KB x CPW) and B, C (16 KB x N).  Every thread keeps its G states in
// registers; the gated output (and, for training, the pre-gate output) leaves straight from
// registers, reduced and stored while the next tile's steps run.  The state entering every
// 16-step chunk is written to chunk_states for the backward pass.
//
// Long sequences with few (batch, channel) tiles are split into S segments: a summary pass
// (mode kModeSummary) scans every segment from a zero state and records its decay product
// and end state, ssm_carry_kernel composes them sequentially per state (the chunk-level
// combine of models/scan.py:160-164), and the main pass rescans each segment from its
// carried-in state.
#pragma once

#include "ssm_common.cuh"

namespace ssm {

// kModeMain: the forward.  kModeSummary: decay product and end state of a segment scanned from
// zero (no outputs).  kModeAdjoint: the reverse adjoint of a segment from a zero adjoint at its
// end, dh_{t-1} = a_t (dh_t + C_t dys_t), giving the gradient with respect to the state entering
// the segment and the decay product (the backward's counterpart of kModeSummary; the u slot
// carries dy, the B slot carries C).
enum { kModeMain = 0, kModeSummary = 1, kModeAdjoint = 2 };

// One warp per CTA.  The CTA owns the CPW channels of one warp; its TMA boxes are BXC channels
// wide (BXC = CPW, widened to 16 bytes of channels when CPW is narrower: the box then starts at
// the 16-byte boundary below the warp's first channel and the warp reads its columns at OFF).
// KB = 16-step tiles per TMA box: fewer, larger TMA requests per step (measured: the forward's
// time falls by 4 % at KB = 2 and 7-9 % at KB = 4 on unsplit sequences; split sequences with short
// segments prefer KB = 2, the smaller ring).
template <int N, int G, typename T, int KB_>
struct FwdSmem {
  static constexpr int TC = 16;
  static constexpr int KB = KB_;                         // 16-step tiles per box
  static constexpr int TB = TC * KB;                     // box rows (time steps)
  static constexpr int CPW = Geo<N, G>::CPW;
  static constexpr int E = (int)sizeof(T);
  static constexpr int BXC = (CPW * E >= 16) ? CPW : 16 / E;
  static constexpr int NSTAGE = KB >= 4 ? 2 : 4 / KB;
  static constexpr int ACT = TB * BXC * E;               // one (TB x BXC) activation box, bytes
  static constexpr int BC = TB * N * E;                  // one (TB x N) box, bytes
  static constexpr int OFF_U = 0, OFF_DT = ACT, OFF_Z = 2 * ACT, OFF_B = 3 * ACT, OFF_C = 3 * ACT + BC;
  static constexpr int STAGE = 3 * ACT + 2 * BC;
  static constexpr int OFF_BAR = NSTAGE * STAGE;
  // the tile's step sizes as fp32 (activated when dt_softplus; bf16 always), and for bf16 its u
  static constexpr int OFF_SDT = OFF_BAR + NSTAGE * 8;
  static constexpr int OFF_SU = OFF_SDT + TC * BXC * 4;
  // bf16: the current box's B and C converted to fp32 once (a lane would otherwise unpack eight bf16
  // values per step); fp32 reads the staged box directly
  static constexpr int OFF_BCF = (OFF_SU + (E == 2 ? TC * BXC * 4 : 0) + 15) / 16 * 16;
  static constexpr int BCF = (E == 2) ? 2 * TB * N * 4 : 0;
  static constexpr int BYTES = OFF_BCF + BCF;
  static_assert(ACT % 128 == 0 && BC % 128 == 0, "TMA boxes must stay 128-byte aligned");
};

// Discretization of one step for a pair of states, split into the state-independent
// coefficients (phase A) and the update (phase B), h' = a h + b for every method.  ZOH:
// b = expm1(dt A) / A * B u with expm1 from em1x2 (accurate also for small |dt A|).

template <int METHOD>
__device__ __forceinline__ void fwd_coeffs2(float2 dt2, float2 u2, float2 dtu2, float2 B2, float2 Ak2, float2 A2k2,
                                            float2 iA2, float2& a, float2& bco) {
  if (METHOD == kZOH) {
    const float2 x = mul2(dt2, A2k2);
    a = ex2x2(x);
    bco = mul2(em1x2(x, a), mul2(mul2(B2, u2), iA2));
  } else if (METHOD == kEuler) {
    a = ex2x2(mul2(dt2, A2k2));
    bco = mul2(dtu2, B2);
  } else {
    const float2 z = mul2(dt2, Ak2);
    const float2 w = rcpx2(fma2(bc2(-0.5f), z, bc2(1.0f)));
    a = mul2(fma2(bc2(0.5f), z, bc2(1.0f)), w);
    bco = mul2(mul2(dtu2, B2), w);
  }
}
template <int METHOD>
__device__ __forceinline__ float2 fwd_apply2(float2 h, float2 a, float2 bco) {
  return fma2(a, h, bco);
}

constexpr int kFwdSub = 4;   // steps per state-independent sub-tile of the forward (divides 16)

template <typename S, int MODE>
__device__ __forceinline__ void fwd_issue_loads(const FwdParams& p, unsigned char* st, uint64_t* bar, int x0,
                                                int t0, int b) {
  const bool load_c = (MODE == kModeMain);
  const bool load_z = (MODE != kModeSummary) && p.has_z;
  const uint32_t tx = 2 * S::ACT + S::BC + (load_c ? S::BC : 0) + (load_z ? S::ACT : 0);
  mbar_arrive_expect_tx(bar, tx);
  tma_load_3d(st + S::OFF_U, &p.tm_u, bar, x0, t0, b);
  tma_load_3d(st + S::OFF_DT, &p.tm_dt, bar, x0, t0, b);
  tma_load_3d(st + S::OFF_B, &p.tm_B, bar, 0, t0, b);
  if (load_c) tma_load_3d(st + S::OFF_C, &p.tm_C, bar, 0, t0, b);
  if (load_z) tma_load_3d(st + S::OFF_Z, &p.tm_z, bar, x0, t0, b);
}

// Plain (non-TMA) box load with zero fill by the warp, for views TMA cannot describe.
template <typename S, int N, typename T, int MODE>
__device__ __forceinline__ void fwd_warp_load(const FwdParams& p, unsigned char* st, int x0, int t0, int b) {
  const T zero = from_f32<T>(0.0f);
  for (int e = threadIdx.x; e < S::TB * S::BXC; e += 32) {
    const int tt = e / S::BXC, dd = e % S::BXC;
    const int t = t0 + tt, dg = x0 + dd;
    const bool ok = t < p.L && dg < p.D;
    const long long tl = t;
    auto ld = [&](const DAct& a) { return ok ? static_cast<const T*>(a.ptr)[b * a.sb + tl * a.sl + dg] : zero; };
    reinterpret_cast<T*>(st + S::OFF_U)[e] = ld(p.u);
    reinterpret_cast<T*>(st + S::OFF_DT)[e] = ld(p.dt);
    if (MODE != kModeSummary && p.has_z) reinterpret_cast<T*>(st + S::OFF_Z)[e] = ld(p.z);
  }
  for (int e = threadIdx.x; e < S::TB * N; e += 32) {
    const int tt = e / N, n = e % N;
    const int t = t0 + tt;
    const bool ok = t < p.L;
    reinterpret_cast<T*>(st + S::OFF_B)[e] =
        ok ? static_cast<const T*>(p.Bm.ptr)[b * p.Bm.sb + (long long)t * p.Bm.sl + n] : zero;
    if (MODE == kModeMain)
      reinterpret_cast<T*>(st + S::OFF_C)[e] =
          ok ? static_cast<const T*>(p.Cm.ptr)[b * p.Cm.sb + (long long)t * p.Cm.sl + n] : zero;
  }
}

// One warp per CTA, no CTA-wide synchronisation: lane 0 keeps an NSTAGE-deep TMA ring of
// 16-step boxes in flight, all lanes wait on the box's mbarrier, and the outputs leave straight
// from registers.  Warps progress independently, so one warp's reductions and stores overlap
// other warps' recurrences.
template <int N, int G, int METHOD, typename T, int MODE, int KB_>
__global__ void __launch_bounds__(32) ssm_fwd_kernel(const __grid_constant__ FwdParams p) {
  using Gm = Geo<N, G>;
  using S = FwdSmem<N, G, T, KB_>;
  constexpr int TC = Gm::TC, LPC = Gm::LPC, CPW = Gm::CPW, BXC = S::BXC;
  constexpr int NP = G / 2;
  constexpr int YPL = TC / LPC;   // output steps per lane after the y reduction
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  pdl_launch_dependents();
  pdl_wait();

  // Lane layout: state group major.  The 8 lanes of a quarter warp then share one state group,
  // so the vector loads of B and C read one address per quarter warp (a broadcast) instead of
  // LPC different ones.
  const int lane = threadIdx.x;
  const int c = lane % CPW, g = lane / CPW;
  constexpr int GSTRIDE = CPW;   // lane distance between a channel's state groups
  const int b = blockIdx.z, seg = blockIdx.y + p.seg_first;
  const int d0 = blockIdx.x * CPW;
  const int x0 = (d0 / BXC) * BXC, dl = d0 - x0 + c;   // box origin and this lane's column
  const int d = d0 + c;
  const bool dvalid = d < p.D;
  const int nbase = g * G;
  const int t_begin = seg * p.seg_len;
  const int t_end = min(p.L, t_begin + p.seg_len);
  const int nblk = (t_end - t_begin + TC - 1) / TC;
  // boxes of KB tiles; the adjoint walks the segment's tiles (and boxes) from the last to the first
  constexpr int KB = S::KB;
  const int nbox = (nblk + KB - 1) / KB;
  auto box_t0 = [&](int q) { return t_begin + ((MODE == kModeAdjoint) ? nbox - 1 - q : q) * S::TB; };

  // Per-state constants, as pairs: A, A log2(e) (for 2^x), 1/A.  Channels past D get A = -1
  // and zero inputs.
  float2 Ak[NP], A2[NP], iA[NP];
  {
    float av[G];
#pragma unroll
    for (int k = 0; k < G; ++k) av[k] = -1.f;
    if (dvalid) loadg<G>(p.A + (size_t)d * N + nbase, av);
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      Ak[i] = make_float2(av[2 * i], av[2 * i + 1]);
      A2[i] = mul2(Ak[i], bc2(kLog2e));
      iA[i] = make_float2(1.0f / av[2 * i], 1.0f / av[2 * i + 1]);
    }
  }
  // D skip, added to the reduced y of the lane's output steps
  const float Dd0 = (MODE == kModeMain && p.Dskip != nullptr && dvalid) ? p.Dskip[d] : 0.0f;

  float2 h[NP], P[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    h[i] = bc2(0.f);
    P[i] = bc2(1.f);
  }
  if (dvalid && MODE != kModeAdjoint) {
    const float* src = nullptr;
    if (p.seg_init != nullptr) src = p.seg_init + (((size_t)b * p.nseg + seg) * p.D + d) * N + nbase;
    else if (seg == 0 && p.h_init != nullptr) src = p.h_init + ((size_t)b * p.D + d) * N + nbase;
    if (src != nullptr) loadp<G>(src, h);
  }

  if (MODE == kModeMain && !p.has_z) {   // z tiles are never loaded: keep them zero
    for (int e = lane; e < S::NSTAGE * S::ACT / 4; e += 32)
      reinterpret_cast<uint32_t*>(smem + (e / (S::ACT / 4)) * S::STAGE + S::OFF_Z)[e % (S::ACT / 4)] = 0u;
  }
  if (p.use_tma) {
    if (lane == 0) {
#pragma unroll
      for (int s = 0; s < S::NSTAGE; ++s) mbar_init(&bars[s], 1);
      fence_mbar_init();
      for (int s = 0; s < S::NSTAGE && s < nbox; ++s)
        fwd_issue_loads<S, MODE>(p, smem + s * S::STAGE, &bars[s], x0, box_t0(s), b);
    }
    __syncwarp();
  }

  T* const yout = static_cast<T*>(const_cast<void*>(p.y.ptr)) + b * p.y.sb + d;
  T* const ygout = static_cast<T*>(const_cast<void*>(p.yg.ptr)) + b * p.yg.sb + d;

  // Output of one box: y over the LPC lanes of each channel (lane g ends with steps g, g + LPC,
  // ...), the gate, and the stores.  tb < 0 marks "no box" (the stores are skipped).
  auto emit = [&](float (&v)[TC], const float (&zz)[TC / LPC], const float (&uu)[TC / LPC], int tb) {
    xpose_reduce<TC, LPC, GSTRIDE>(v, lane);
#pragma unroll
    for (int i = 0; i < YPL; ++i) {
      const int t = tb + g + i * LPC;
      const float yv = fmaf(Dd0, uu[i], v[i]);
      // the gate as a select and predicated stores: no branch inside the step loop this runs in
      const float yo = p.has_z ? yv * (zz[i] * sigmoid(zz[i])) : yv;
      const bool ok = tb >= 0 && dvalid && t < p.L;
      // 4-tile boxes (grids that fit the GPU at once, few warps per SM): predicated stores keep the
      // step loop one basic block for the scheduler (config 1 forward 59.0 -> 54.1 us); 2-tile boxes
      // (many warps per SM) keep branches (config 2: 1.09 vs 1.15 ms, config 3: 3.40 vs 3.48 ms)
      if constexpr (KB >= 4) {
        st_pred(ygout + (long long)t * p.yg.sl, from_f32<T>(yv), ok && p.save_ygate);
        st_pred(yout + (long long)t * p.y.sl, from_f32<T>(yo), ok);
      } else {
        if (ok && p.save_ygate) ygout[(long long)t * p.yg.sl] = from_f32<T>(yv);
        if (ok) yout[(long long)t * p.y.sl] = from_f32<T>(yo);
      }
    }
  };
  // the previous tile's outputs wait here and are emitted from inside the next tile's step loop,
  // so their shuffles, MUFU work and stores overlap the recurrence
  float ypv[TC], zpv[TC / LPC], upv[TC / LPC];
  int tpv = -1;
#pragma unroll
  for (int i = 0; i < TC; ++i) ypv[i] = 0.f;
#pragma unroll
  for (int i = 0; i < TC / LPC; ++i) zpv[i] = upv[i] = 0.f;

  // Two tiles per loop trip: the hand-over of a tile's outputs to the next trip (ypv = yp, ...)
  // then becomes register renaming instead of 24 moves per tile (96 -> 114 registers; config 1
  // forward 49.25 -> 47.3 us, step 171.1 -> 169.2 us, same box).
#pragma unroll 2
  for (int k = 0; k < nblk; ++k) {
    const int tix = (MODE == kModeAdjoint) ? nblk - 1 - k : k;     // tile within the segment
    const int bx = tix / KB, sub = tix % KB;
    const int q = (MODE == kModeAdjoint) ? nbox - 1 - bx : bx;      // box in processing order
    const bool first_in_box = (MODE == kModeAdjoint) ? (tix == nblk - 1 || sub == KB - 1) : sub == 0;
    const bool last_in_box = (MODE == kModeAdjoint) ? sub == 0 : (sub == KB - 1 || tix == nblk - 1);
    const int s = q % S::NSTAGE;
    const int t0 = t_begin + tix * TC;
    unsigned char* st = smem + s * S::STAGE;
    if (first_in_box) {
      if (p.use_tma) {
        mbar_wait(&bars[s], (uint32_t)((q / S::NSTAGE) & 1), p.err);
      } else {
        __syncwarp();
        fwd_warp_load<S, N, T, MODE>(p, st, x0, box_t0(q), b);
        __syncwarp();
      }
      if constexpr (sizeof(T) == 2) {   // the box's B (and C) as fp32: 8 values per 16-byte load
        constexpr int NV = S::TB * N / 8;
        float4* const dst = reinterpret_cast<float4*>(smem + S::OFF_BCF);
        const uint4* const srcB = reinterpret_cast<const uint4*>(st + S::OFF_B);
        const uint4* const srcC = reinterpret_cast<const uint4*>(st + S::OFF_C);
        auto widen = [&](const uint4* src, float4* out, int v) {
          const uint4 w = src[v];
          out[2 * v] = make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u),
                                   __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
          out[2 * v + 1] = make_float4(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xffff0000u),
                                       __uint_as_float(w.w << 16), __uint_as_float(w.w & 0xffff0000u));
        };
#pragma unroll
        for (int v = lane; v < NV; v += 32) {
          widen(srcB, dst, v);
          if (MODE == kModeMain) widen(srcC, dst + NV * 2, v);
        }
        __syncwarp();
      }
    }
    // this tile's rows of the box
    const T* __restrict__ Xs = reinterpret_cast<const T*>(st + S::OFF_U) + sub * TC * BXC;
    const T* __restrict__ DLs = reinterpret_cast<const T*>(st + S::OFF_DT) + sub * TC * BXC;
    const T* __restrict__ Zs = reinterpret_cast<const T*>(st + S::OFF_Z) + sub * TC * BXC;
    // B and C of this tile's rows as fp32 (bf16: the widened copies of the box)
    const float* __restrict__ Bs = (sizeof(T) == 2 ? reinterpret_cast<const float*>(smem + S::OFF_BCF)
                                                   : reinterpret_cast<const float*>(st + S::OFF_B)) + sub * TC * N;
    const float* __restrict__ Cs = (sizeof(T) == 2 ? reinterpret_cast<const float*>(smem + S::OFF_BCF) + S::TB * N
                                                   : reinterpret_cast<const float*>(st + S::OFF_C)) + sub * TC * N;

    if (MODE == kModeMain && p.chunk_states != nullptr && dvalid)   // state entering chunk t0 / 16
      storep<G>(p.chunk_states + (((size_t)b * p.nchunks + t0 / TC) * p.D + d) * N + nbase, h);

    // The tile's deltas go once per element into an fp32 tile: activated, softplus(raw + bias), when
    // dt_softplus (rows past L and columns past D stay 0: identity steps), else (bf16) converted; bf16
    // also converts u.  The step loop then reads fp32 without per-step conversions (each value is
    // read by the LPC lanes of its channel).  The previous tile's readers are done: every lane
    // passed the __syncwarp at the end of that tile.
    float* const SDT = reinterpret_cast<float*>(smem + S::OFF_SDT);
    float* const SU = reinterpret_cast<float*>(smem + S::OFF_SU);
    if (p.dt_softplus || sizeof(T) == 2) {
      for (int e = lane; e < TC * BXC; e += 32) {
        const int t = t0 + e / BXC, dg = x0 + e % BXC;
        const float raw = to_f32(DLs[e]);
        SDT[e] = !p.dt_softplus ? raw
                 : (t < p.L && dg < p.D) ? softplus(raw + (p.dt_bias != nullptr ? p.dt_bias[dg] : 0.0f))
                                         : 0.0f;
        if constexpr (sizeof(T) == 2) SU[e] = to_f32(Xs[e]);
      }
      __syncwarp();
    }
    // the step sizes this tile reads: the activated tile, or the raw box (fp32: one pointer, chosen
    // once per tile, so the unrolled step loop stays one basic block)
    const float* const dsrc = (sizeof(T) == 4 && !p.dt_softplus) ? reinterpret_cast<const float*>(DLs) : SDT;
    auto delta_at = [&](int i) -> float {
      if constexpr (sizeof(T) == 4) {
        return dsrc[i];
      } else {
        return SDT[i];
      }
    };
    auto u_at = [&](int i) -> float {   // u (the adjoint pass: dy)
      if constexpr (sizeof(T) == 4) {
        return Xs[i];
      } else {
        return SU[i];
      }
    };

    float yp[TC], zk[YPL], uk[YPL];   // main mode: partial y; the gate's z and the D-skip u of the lane's output steps
    if constexpr (MODE == kModeAdjoint) {
      // reverse through the box: dh <- a_t dh + a_t C_t dys_t, dys = dy silu(z) (or dy)
#pragma unroll
      for (int t0s = TC - kFwdSub; t0s >= 0; t0s -= kFwdSub) {
        float2 av[kFwdSub][NP], cd[kFwdSub][NP];
#pragma unroll
        for (int q = 0; q < kFwdSub; ++q) {
          const int tt = t0s + q;
          float dys = u_at(tt * BXC + dl);
          const float dtv = delta_at(tt * BXC + dl);
          if (p.has_z) {
            const float zz = to_f32(Zs[tt * BXC + dl]);
            dys *= zz * sigmoid(zz);
          }
          const float2 dt2 = bc2(dtv), dys2 = bc2(dys);
          float2 Cn[NP];
          loadp<G>(Bs + tt * N + nbase, Cn);
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            float2 unused;
            fwd_coeffs2<METHOD>(dt2, bc2(0.f), bc2(0.f), Cn[i], Ak[i], A2[i], iA[i], av[q][i], unused);
            cd[q][i] = mul2(av[q][i], mul2(Cn[i], dys2));
          }
        }
#pragma unroll
        for (int q = kFwdSub - 1; q >= 0; --q) {
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            h[i] = fma2(av[q][i], h[i], cd[q][i]);
            P[i] = mul2(P[i], av[q][i]);
          }
        }
      }
    } else {
      // 16 steps.  The lane's partial y (over its G states) stays in registers, stored at
      // yp[(t % LPC) YPL + t / LPC] so that after the reduction lane g holds steps g, g + LPC, ...;
      // the lane also keeps z and u of those steps (read after the step loop).  Steps are
      // processed in sub-tiles: phase A computes what does not depend on the state (decays,
      // inputs, C), phase B is only the recurrence and the y accumulation.  The next sub-tile's
      // inputs are fetched from shared memory before this one's coefficients are computed, so the
      // loads' latency overlaps the work.
      float fu[2][kFwdSub], fdt[2][kFwdSub];
      float2 fB[2][kFwdSub][NP], fC[2][kFwdSub][NP];
      auto fetch = [&](int slot, int base) {
#pragma unroll
        for (int q = 0; q < kFwdSub; ++q) {
          const int tt = base + q;
          fu[slot][q] = u_at(tt * BXC + dl);
          fdt[slot][q] = delta_at(tt * BXC + dl);
          loadp<G>(Bs + tt * N + nbase, fB[slot][q]);
          if (MODE == kModeMain) loadp<G>(Cs + tt * N + nbase, fC[slot][q]);
        }
      };
      fetch(0, 0);
#pragma unroll
      for (int t0s = 0; t0s < TC; t0s += kFwdSub) {
        const int cur = (t0s / kFwdSub) & 1;
        if (t0s + kFwdSub < TC) fetch(cur ^ 1, t0s + kFwdSub);
        float2 av[kFwdSub][NP], bv[kFwdSub][NP], cv[kFwdSub][NP];
#pragma unroll
        for (int q = 0; q < kFwdSub; ++q) {
          const float uu = fu[cur][q];
          const float dtv = fdt[cur][q];
          const float2 u2 = bc2(uu), dt2 = bc2(dtv), dtu2 = bc2(dtv * uu);
          float2 Bn[NP];
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            Bn[i] = fB[cur][q][i];
            cv[q][i] = fC[cur][q][i];
          }
#pragma unroll
          for (int i = 0; i < NP; ++i)
            fwd_coeffs2<METHOD>(dt2, u2, dtu2, Bn[i], Ak[i], A2[i], iA[i], av[q][i], bv[q][i]);
        }
#pragma unroll
        for (int q = 0; q < kFwdSub; ++q) {
          const int tt = t0s + q;
          float2 acc = bc2(0.f);
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            h[i] = fwd_apply2<METHOD>(h[i], av[q][i], bv[q][i]);
            if (MODE == kModeMain) acc = (i == 0) ? mul2(cv[q][i], h[i]) : fma2(cv[q][i], h[i], acc);
            else P[i] = mul2(P[i], av[q][i]);
          }
          yp[(tt % LPC) * YPL + tt / LPC] = acc.x + acc.y;
        }
        if (MODE == kModeMain && t0s == (TC > kFwdSub ? kFwdSub : 0)) emit(ypv, zpv, upv, tpv);
      }
      if (MODE == kModeMain) {   // z and u of the lane's output steps, before the refill
#pragma unroll
        for (int i = 0; i < YPL; ++i) {
          zk[i] = to_f32(Zs[(g + i * LPC) * BXC + dl]);
          uk[i] = u_at((g + i * LPC) * BXC + dl);
        }
      }
    }
    // every lane has read this tile (and the activated-delta tile); after a box's last tile the
    // stage goes back to the TMA ring
    __syncwarp();
    if (last_in_box && p.use_tma && lane == 0 && q + S::NSTAGE < nbox)
      fwd_issue_loads<S, MODE>(p, st, &bars[s], x0, box_t0(q + S::NSTAGE), b);

    if (MODE == kModeMain) {
#pragma unroll
      for (int i = 0; i < TC; ++i) ypv[i] = yp[i];
#pragma unroll
      for (int i = 0; i < YPL; ++i) {
        zpv[i] = zk[i];
        upv[i] = uk[i];
      }
      tpv = t0;
    }
  }

  if (MODE == kModeMain) {
    emit(ypv, zpv, upv, tpv);
    if (dvalid && t_end == p.L && p.last != nullptr) storep<G>(p.last + ((size_t)b * p.D + d) * N + nbase, h);
  } else if (dvalid) {
    const size_t o = (((size_t)b * p.nseg + seg) * p.D + d) * N + nbase;
    storep<G>(p.seg_hend + o, h);
    storep<G>(p.seg_decay + o, P);
  }
}

// Host-side launcher (defined per element type in ssm_fwd_<type>.cu).  G = states per thread.
template <typename T>
cudaError_t launch_fwd(int N, int G, int method, int mode, int kb, const FwdParams& p, dim3 grid, cudaStream_t stream);
template <typename T>
int fwd_smem_bytes(int N, int G, int kb);

}  // namespace ssm
