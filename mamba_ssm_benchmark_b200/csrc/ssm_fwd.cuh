// ssm_fwd.cuh — forward selective scan on sm_100a.
//
// Replaces the reference's forward GPU path, kernels/triton_scan.py:27-74 (_fwd_kernel) and
// :253-286 (_launch_fwd, TritonSelectiveScanFn.forward); the math is models/scan.py:39-55
// (discretize) and :70-76 (the recurrence h_t = a_t h_{t-1} + b_t), y_t = <C_t, h_t>.
//
// One CTA owns a (batch, 32-channel tile, time segment).  The CTA walks its segment in tiles
// of 16 steps; thread 0 streams u, delta, z (16 x 32) and B, C (16 x N) tiles through a
// 3-stage TMA ring (mbarrier completion), every thread keeps its G states in registers, and
// the gated output tile (and, for training, the pre-gate tile) goes back to HBM through a
// bank-conflict-free padded shared tile and coalesced 16-byte stores.  The state entering every 16-step chunk is written to chunk_states for the
// backward pass.
//
// Long sequences with few (batch, channel) tiles are split into S segments: a summary pass
// (mode kModeSummary) scans every segment from a zero state and records its decay product
// and end state, ssm_carry_kernel composes them sequentially per state (the chunk-level
// combine of models/scan.py:160-164), and the main pass rescans each segment from its
// carried-in state.
#pragma once

#include "ssm_common.cuh"

namespace ssm {

enum { kModeMain = 0, kModeSummary = 1 };

template <int N, int G, typename T>
struct FwdSmem {
  static constexpr int TC = 16, DT = 32;
  static constexpr int NSTAGE = 3;
  static constexpr int NOUT = 2;
  static constexpr int ACT = TC * DT * (int)sizeof(T);   // one dense (16 x 32) TMA tile, bytes
  static constexpr int BC = TC * N * (int)sizeof(T);     // one (16 x N) tile, bytes
  // Output tiles use a padded row pitch: the epilogue writes (step, channel) blocks of
  // LPC rows x CPW channels, which the pitch spreads over the 32 banks.
  static constexpr int OP = PadPitch<Geo<N, G>::CPW, T>::value;
  static constexpr int OUT = ((TC * OP * (int)sizeof(T)) + 127) / 128 * 128;
  static constexpr int OFF_U = 0, OFF_DT = ACT, OFF_Z = 2 * ACT, OFF_B = 3 * ACT, OFF_C = 3 * ACT + BC;
  static constexpr int STAGE = 3 * ACT + 2 * BC;
  static constexpr int OFF_Y = NSTAGE * STAGE;             // NOUT x {y, pre-gate y}
  static constexpr int OFF_BAR = OFF_Y + NOUT * 2 * OUT;
  static constexpr int BYTES = OFF_BAR + NSTAGE * 8;
  static_assert(ACT % 128 == 0 && BC % 128 == 0, "TMA tiles must stay 128-byte aligned");
};

// Discretization of one (step, state) split into the state-independent coefficients and the
// update.  ZOH: b = expm1(dt A)/A B u is applied as h' = a (h + g) - g with g = B u / A, i.e.
// the coefficient pair is (a, g); Euler and bilinear use h' = a h + b.
template <int METHOD>
__device__ __forceinline__ void fwd_coeffs(float dtv, float uu, float dtu, float Bn, float Ak, float A2, float iA,
                                           float& a, float& bcoef) {
  if (METHOD == kZOH) {
    a = ex2(dtv * A2);
    bcoef = (Bn * uu) * iA;
  } else if (METHOD == kEuler) {
    a = ex2(dtv * A2);
    bcoef = dtu * Bn;
  } else {
    const float z = dtv * Ak;
    const float w = rcp(fmaf(-0.5f, z, 1.0f));
    a = fmaf(0.5f, z, 1.0f) * w;
    bcoef = (dtu * Bn) * w;
  }
}
template <int METHOD>
__device__ __forceinline__ float fwd_apply(float h, float a, float bcoef) {
  if (METHOD == kZOH) return fmaf(a, h + bcoef, -bcoef);
  return fmaf(a, h, bcoef);
}

#ifndef SSM_FWD_SUB
#define SSM_FWD_SUB 4   // steps per state-independent sub-tile (divides 16)
#endif

template <typename S, int MODE>
__device__ __forceinline__ void fwd_issue_loads(const FwdParams& p, unsigned char* st, uint64_t* bar, int d0,
                                                int t0, int b) {
  const bool load_zc = (MODE == kModeMain);
  const uint32_t tx = 2 * S::ACT + S::BC + (load_zc ? (S::BC + (p.has_z ? S::ACT : 0)) : 0);
  mbar_arrive_expect_tx(bar, tx);
  tma_load_3d(st + S::OFF_U, &p.tm_u, bar, d0, t0, b);
  tma_load_3d(st + S::OFF_DT, &p.tm_dt, bar, d0, t0, b);
  tma_load_3d(st + S::OFF_B, &p.tm_B, bar, 0, t0, b);
  if (load_zc) {
    tma_load_3d(st + S::OFF_C, &p.tm_C, bar, 0, t0, b);
    if (p.has_z) tma_load_3d(st + S::OFF_Z, &p.tm_z, bar, d0, t0, b);
  }
}

// Cooperative (non-TMA) tile load with zero fill, for views TMA cannot describe.
template <typename S, int N, int NT, typename T, int MODE>
__device__ __forceinline__ void fwd_coop_load(const FwdParams& p, unsigned char* st, int d0, int t0, int b) {
  const T zero = from_f32<T>(0.0f);
  for (int e = threadIdx.x; e < S::TC * S::DT; e += NT) {
    const int tt = e / S::DT, dd = e % S::DT;
    const int t = t0 + tt, dg = d0 + dd;
    const bool ok = t < p.L && dg < p.D;
    const long long tl = t;
    auto ld = [&](const DAct& a) { return ok ? static_cast<const T*>(a.ptr)[b * a.sb + tl * a.sl + dg] : zero; };
    reinterpret_cast<T*>(st + S::OFF_U)[e] = ld(p.u);
    reinterpret_cast<T*>(st + S::OFF_DT)[e] = ld(p.dt);
    if (MODE == kModeMain && p.has_z) reinterpret_cast<T*>(st + S::OFF_Z)[e] = ld(p.z);
  }
  for (int e = threadIdx.x; e < S::TC * N; e += NT) {
    const int tt = e / N, n = e % N;
    const int t = t0 + tt;
    const bool ok = t < p.L;
    const T* Bm = static_cast<const T*>(p.Bm.ptr);
    reinterpret_cast<T*>(st + S::OFF_B)[e] = ok ? Bm[b * p.Bm.sb + (long long)t * p.Bm.sl + n] : zero;
    if (MODE == kModeMain) {
      const T* Cm = static_cast<const T*>(p.Cm.ptr);
      reinterpret_cast<T*>(st + S::OFF_C)[e] = ok ? Cm[b * p.Cm.sb + (long long)t * p.Cm.sl + n] : zero;
    }
  }
}

template <int N, int G, int METHOD, typename T, int MODE>
__global__ void __launch_bounds__(Geo<N, G>::NT) ssm_fwd_kernel(const __grid_constant__ FwdParams p) {
  using Gm = Geo<N, G>;
  using S = FwdSmem<N, G, T>;
  constexpr int TC = Gm::TC, DT = Gm::DT, LPC = Gm::LPC, NT = Gm::NT, OP = S::OP;
  constexpr int YPL = TC / LPC;   // output steps per lane after the y reduction
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = lane / LPC, g = lane % LPC;
  const int dl = warp * Gm::CPW + c;
  const int b = blockIdx.z, seg = blockIdx.y;
  const int d0 = blockIdx.x * DT, d = d0 + dl;
  const bool dvalid = d < p.D;
  const int nbase = g * G;
  const int t_begin = seg * p.seg_len;
  const int t_end = min(p.L, t_begin + p.seg_len);
  const int nblk = (t_end - t_begin + TC - 1) / TC;

  // Per-state constants: A, A log2(e) (for 2^x), 1/A.  Channels past D get A = -1, zero inputs.
  float Ak[G], A2[G], iA[G];
  {
    float av[G];
#pragma unroll
    for (int k = 0; k < G; ++k) av[k] = -1.f;
    if (dvalid) loadg<G>(p.A + (size_t)d * N + nbase, av);
#pragma unroll
    for (int k = 0; k < G; ++k) {
      Ak[k] = av[k];
      A2[k] = av[k] * kLog2e;
      iA[k] = 1.0f / av[k];
    }
  }
  // D skip folded into the partial sum of lane g == 0 of each channel group
  const float Dd0 = (MODE == kModeMain && p.Dskip != nullptr && dvalid && g == 0) ? p.Dskip[d] : 0.0f;

  float h[G], P[G];
#pragma unroll
  for (int k = 0; k < G; ++k) {
    h[k] = 0.f;
    P[k] = 1.f;
  }
  if (dvalid) {
    const float* src = nullptr;
    if (p.seg_init != nullptr) src = p.seg_init + (((size_t)b * p.nseg + seg) * p.D + d) * N + nbase;
    else if (seg == 0 && p.h_init != nullptr) src = p.h_init + ((size_t)b * p.D + d) * N + nbase;
    if (src != nullptr) loadg<G>(src, h);
  }

  if (p.use_tma) {
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < S::NSTAGE; ++s) mbar_init(&bars[s], 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
      for (int s = 0; s < S::NSTAGE && s < nblk; ++s)
        fwd_issue_loads<S, MODE>(p, smem + s * S::STAGE, &bars[s], d0, t_begin + s * TC, b);
    }
  }

  for (int ib = 0; ib < nblk; ++ib) {
    const int s = ib % S::NSTAGE;
    const int t0 = t_begin + ib * TC;
    unsigned char* st = smem + s * S::STAGE;
    if (p.use_tma) {
      mbar_wait(&bars[s], (uint32_t)((ib / S::NSTAGE) & 1), p.err);
    } else {
      fwd_coop_load<S, N, NT, T, MODE>(p, st, d0, t0, b);
      __syncthreads();
    }
    const T* __restrict__ Xs = reinterpret_cast<const T*>(st + S::OFF_U);
    const T* __restrict__ DLs = reinterpret_cast<const T*>(st + S::OFF_DT);
    const T* __restrict__ Zs = reinterpret_cast<const T*>(st + S::OFF_Z);
    const T* __restrict__ Bs = reinterpret_cast<const T*>(st + S::OFF_B);
    const T* __restrict__ Cs = reinterpret_cast<const T*>(st + S::OFF_C);
    T* Ys = reinterpret_cast<T*>(smem + S::OFF_Y + (ib % S::NOUT) * 2 * S::OUT);
    T* YGs = reinterpret_cast<T*>(smem + S::OFF_Y + (ib % S::NOUT) * 2 * S::OUT + S::OUT);

    if (MODE == kModeMain && p.chunk_states != nullptr && dvalid)   // state entering chunk t0 / 16
      storeg<G>(p.chunk_states + (((size_t)b * p.nchunks + t0 / TC) * p.D + d) * N + nbase, h);

    // 16 steps.  The lane's partial y (its G states, plus D u on lane 0 of the group) stays
    // in registers, stored at yp[(t % LPC) YPL + t / LPC] so that after the reduction lane g
    // holds steps g, g + LPC, ...; the lane also keeps z of those steps.
    float yp[TC], zk[YPL];
    // Steps are processed in sub-tiles of SUB: phase A computes everything that does not
    // depend on the state (decays a, inputs b, C) for SUB steps at once, so the MUFU work of
    // a sub-tile runs back to back; phase B is only the recurrence and the y accumulation.
#pragma unroll
    for (int t0s = 0; t0s < TC; t0s += SSM_FWD_SUB) {
      float av[SSM_FWD_SUB][G], bv[SSM_FWD_SUB][G], cv[SSM_FWD_SUB][G], yd[SSM_FWD_SUB];
#pragma unroll
      for (int q = 0; q < SSM_FWD_SUB; ++q) {
        const int tt = t0s + q;
        const float uu = to_f32(Xs[tt * DT + dl]);
        const float dtv = to_f32(DLs[tt * DT + dl]);
        const float dtu = dtv * uu;
        float Bn[G];
        loadg<G>(Bs + tt * N + nbase, Bn);
        if (MODE == kModeMain) loadg<G>(Cs + tt * N + nbase, cv[q]);
        yd[q] = Dd0 * uu;
#pragma unroll
        for (int k = 0; k < G; ++k) fwd_coeffs<METHOD>(dtv, uu, dtu, Bn[k], Ak[k], A2[k], iA[k], av[q][k], bv[q][k]);
        if (MODE == kModeMain && p.has_z) {
          const float zz = to_f32(Zs[tt * DT + dl]);
          if (g == tt % LPC) zk[tt / LPC] = zz;
        }
      }
#pragma unroll
      for (int q = 0; q < SSM_FWD_SUB; ++q) {
        const int tt = t0s + q;
        float acc0 = yd[q], acc1 = 0.f;
#pragma unroll
        for (int k = 0; k < G; ++k) {
          h[k] = fwd_apply<METHOD>(h[k], av[q][k], bv[q][k]);
          if (MODE == kModeMain) {
            if (k & 1) acc1 = fmaf(cv[q][k], h[k], acc1);
            else acc0 = fmaf(cv[q][k], h[k], acc0);
          } else {
            P[k] *= av[q][k];
          }
        }
        yp[(tt % LPC) * YPL + tt / LPC] = acc0 + acc1;
      }
    }
    if (MODE == kModeMain) {
      xpose_reduce<TC, LPC, 1>(yp, lane);
#pragma unroll
      for (int i = 0; i < YPL; ++i) {
        const int tt = g + i * LPC;
        float yv = yp[i];
        if (p.save_ygate) YGs[tt * OP + dl] = from_f32<T>(yv);
        if (p.has_z) yv *= zk[i] * sigmoid(zk[i]);
        Ys[tt * OP + dl] = from_f32<T>(yv);
      }
    }
    __syncthreads();
    if (MODE == kModeMain) {
      store_tile<NT, OP>(Ys, p.y, b, t0, d0, p.L, p.D);
      if (p.save_ygate) store_tile<NT, OP>(YGs, p.yg, b, t0, d0, p.L, p.D);
    }
    if (p.use_tma && tid == 0 && ib + S::NSTAGE < nblk)
      fwd_issue_loads<S, MODE>(p, st, &bars[s], d0, t0 + S::NSTAGE * TC, b);
  }

  if (MODE == kModeMain) {
    if (dvalid && t_end == p.L && p.last != nullptr) storeg<G>(p.last + ((size_t)b * p.D + d) * N + nbase, h);
  } else if (dvalid) {
    const size_t o = (((size_t)b * p.nseg + seg) * p.D + d) * N + nbase;
    storeg<G>(p.seg_hend + o, h);
    storeg<G>(p.seg_decay + o, P);
  }
}

// Host-side launcher (defined per element type in ssm_fwd_<type>.cu).  G = states per thread.
template <typename T>
cudaError_t launch_fwd(int N, int G, int method, int mode, const FwdParams& p, dim3 grid, cudaStream_t stream);

}  // namespace ssm
