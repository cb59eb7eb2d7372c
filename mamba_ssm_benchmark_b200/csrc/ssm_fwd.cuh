// ssm_fwd.cuh — forward selective scan on sm_100a.
//
// Replaces the reference's forward GPU path, kernels/triton_scan.py:27-74 (_fwd_kernel) and
// :253-286 (_launch_fwd, TritonSelectiveScanFn.forward); the math is models/scan.py:39-55
// (discretize) and :70-76 (the recurrence h_t = a_t h_{t-1} + b_t), y_t = <C_t, h_t>.
//
// One CTA owns a (batch, 32-channel tile, time segment).  The CTA walks its segment in tiles
// of 16 steps; thread 0 streams u, delta, z (16 x 32) and B, C (16 x N) tiles through a
// 3-stage TMA ring (mbarrier completion), every thread keeps its 4 states in registers, and
// the gated output tile goes back to HBM with a TMA store.  The state entering every 16-step
// chunk is written to chunk_states for the backward pass.
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

template <int N, typename T>
struct FwdSmem {
  using Gm = Geo<N>;
  static constexpr int NSTAGE = 3;
  static constexpr int NOUT = 3;
  static constexpr int ACT = Gm::TC * Gm::DT * (int)sizeof(T);   // one (16 x 32) tile, bytes
  static constexpr int BC = Gm::TC * N * (int)sizeof(T);          // one (16 x N) tile, bytes
  static constexpr int OFF_U = 0, OFF_DT = ACT, OFF_Z = 2 * ACT, OFF_B = 3 * ACT, OFF_C = 3 * ACT + BC;
  static constexpr int STAGE = 3 * ACT + 2 * BC;
  static constexpr int OFF_Y = NSTAGE * STAGE;
  static constexpr int OFF_BAR = OFF_Y + NOUT * ACT;
  static constexpr int BYTES = OFF_BAR + NSTAGE * 8;
  static_assert(ACT % 128 == 0 && BC % 128 == 0, "TMA tiles must stay 128-byte aligned");
};

// One time step of one state for the forward recurrence (discretize + update).
template <int METHOD>
__device__ __forceinline__ float fwd_step(float h, float dtv, float uu, float dtu, float Bn, float Ak, float A2,
                                          float iA, float& a_out) {
  if (METHOD == kZOH) {
    // b = expm1(dt A)/A * B u  ->  h' = a h + (a - 1) g  with g = B u / A  = a (h + g) - g
    const float a = ex2(dtv * A2);
    const float gg = (Bn * uu) * iA;
    a_out = a;
    return fmaf(a, h + gg, -gg);
  } else if (METHOD == kEuler) {
    const float a = ex2(dtv * A2);
    a_out = a;
    return fmaf(a, h, dtu * Bn);
  } else {
    const float z = dtv * Ak;
    const float w = rcp(fmaf(-0.5f, z, 1.0f));
    const float a = fmaf(0.5f, z, 1.0f) * w;
    a_out = a;
    return fmaf(a, h, (dtu * Bn) * w);
  }
}

template <int N, typename T, int MODE>
__device__ __forceinline__ void fwd_issue_loads(const FwdParams& p, unsigned char* st, uint64_t* bar, int d0,
                                                int t0, int b) {
  using S = FwdSmem<N, T>;
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
template <int N, typename T, int MODE>
__device__ __forceinline__ void fwd_coop_load(const FwdParams& p, unsigned char* st, int d0, int t0, int b) {
  using Gm = Geo<N>;
  using S = FwdSmem<N, T>;
  const T zero = from_f32<T>(0.0f);
  for (int e = threadIdx.x; e < Gm::TC * Gm::DT; e += Gm::NT) {
    const int tt = e / Gm::DT, dd = e % Gm::DT;
    const int t = t0 + tt, dg = d0 + dd;
    const bool ok = t < p.L && dg < p.D;
    const T* u = static_cast<const T*>(p.u.ptr);
    const T* dt = static_cast<const T*>(p.dt.ptr);
    reinterpret_cast<T*>(st + S::OFF_U)[e] = ok ? u[b * p.u.sb + (long long)t * p.u.sl + dg] : zero;
    reinterpret_cast<T*>(st + S::OFF_DT)[e] = ok ? dt[b * p.dt.sb + (long long)t * p.dt.sl + dg] : zero;
    if (MODE == kModeMain && p.has_z) {
      const T* z = static_cast<const T*>(p.z.ptr);
      reinterpret_cast<T*>(st + S::OFF_Z)[e] = ok ? z[b * p.z.sb + (long long)t * p.z.sl + dg] : zero;
    }
  }
  for (int e = threadIdx.x; e < Gm::TC * N; e += Gm::NT) {
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

template <int N, int METHOD, typename T, int MODE>
__global__ void __launch_bounds__(Geo<N>::NT) ssm_fwd_kernel(const __grid_constant__ FwdParams p) {
  using Gm = Geo<N>;
  using S = FwdSmem<N, T>;
  constexpr int TC = Gm::TC, DT = Gm::DT, LPC = Gm::LPC, TG = LPC;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = lane / LPC, g = lane % LPC;
  const int dl = warp * Gm::CPW + c;
  const int b = blockIdx.z, seg = blockIdx.y;
  const int d0 = blockIdx.x * DT, d = d0 + dl;
  const bool dvalid = d < p.D;
  const int t_begin = seg * p.seg_len;
  const int t_end = min(p.L, t_begin + p.seg_len);
  const int nblk = (t_end - t_begin + TC - 1) / TC;

  // Per-state constants: A, A log2(e) (for 2^x), 1/A.  Channels past D get A = -1, zero inputs.
  float Ak[4], A2[4], iA[4];
  {
    float a4[4] = {-1.f, -1.f, -1.f, -1.f};
    if (dvalid) load4(p.A + (size_t)d * N + g * 4, a4);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      Ak[k] = a4[k];
      A2[k] = a4[k] * kLog2e;
      iA[k] = 1.0f / a4[k];
    }
  }
  const float Dd = (MODE == kModeMain && p.Dskip != nullptr && dvalid) ? p.Dskip[d] : 0.0f;

  float h[4] = {0.f, 0.f, 0.f, 0.f};
  float P[4] = {1.f, 1.f, 1.f, 1.f};
  if (dvalid) {
    const float* src = nullptr;
    if (p.seg_init != nullptr) src = p.seg_init + (((size_t)b * p.nseg + seg) * p.D + d) * N + g * 4;
    else if (seg == 0 && p.h_init != nullptr) src = p.h_init + ((size_t)b * p.D + d) * N + g * 4;
    if (src != nullptr) load4(src, h);
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
        fwd_issue_loads<N, T, MODE>(p, smem + s * S::STAGE, &bars[s], d0, t_begin + s * TC, b);
    }
  }

  for (int ib = 0; ib < nblk; ++ib) {
    const int s = ib % S::NSTAGE;
    const int t0 = t_begin + ib * TC;
    unsigned char* st = smem + s * S::STAGE;
    if (p.use_tma) {
      mbar_wait(&bars[s], (uint32_t)((ib / S::NSTAGE) & 1), p.err);
    } else {
      fwd_coop_load<N, T, MODE>(p, st, d0, t0, b);
      __syncthreads();
    }
    const T* Xs = reinterpret_cast<const T*>(st + S::OFF_U);
    const T* DLs = reinterpret_cast<const T*>(st + S::OFF_DT);
    const T* Zs = reinterpret_cast<const T*>(st + S::OFF_Z);
    const T* Bs = reinterpret_cast<const T*>(st + S::OFF_B);
    const T* Cs = reinterpret_cast<const T*>(st + S::OFF_C);
    T* Ys = reinterpret_cast<T*>(smem + S::OFF_Y + (ib % S::NOUT) * S::ACT);

    if (MODE == kModeMain && p.chunk_states != nullptr && dvalid) {
      // state entering chunk t0 / 16 (t0 is a multiple of 16)
      *reinterpret_cast<float4*>(p.chunk_states + (((size_t)b * p.nchunks + t0 / TC) * p.D + d) * N + g * 4) =
          make_float4(h[0], h[1], h[2], h[3]);
    }

#pragma unroll
    for (int tg = 0; tg < TC; tg += TG) {
      float yp[TG];
#pragma unroll
      for (int j = 0; j < TG; ++j) {
        const int tt = tg + j;
        const float uu = to_f32(Xs[tt * DT + dl]);
        const float dtv = to_f32(DLs[tt * DT + dl]);
        const float dtu = dtv * uu;
        float Bn[4], Cn[4];
        load4(Bs + tt * N + g * 4, Bn);
        if (MODE == kModeMain) load4(Cs + tt * N + g * 4, Cn);
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float a;
          h[k] = fwd_step<METHOD>(h[k], dtv, uu, dtu, Bn[k], Ak[k], A2[k], iA[k], a);
          if (MODE == kModeMain) acc = fmaf(Cn[k], h[k], acc);
          else P[k] *= a;
        }
        yp[j] = acc;
      }
      if (MODE == kModeMain) {
        // y over the LPC lanes of the channel: lane g ends with timestep tg + g
        xpose_reduce<TG, LPC, 1>(yp, lane);
        const int tt = tg + g;
        float yv = yp[0];
        if (p.Dskip != nullptr) yv = fmaf(Dd, to_f32(Xs[tt * DT + dl]), yv);
        if (p.has_z) {
          const float zz = to_f32(Zs[tt * DT + dl]);
          yv *= zz * sigmoid(zz);
        }
        Ys[tt * DT + dl] = from_f32<T>(yv);
      }
    }

    if (p.use_tma) {
      fence_proxy_async_smem();
      // the store that last read the output buffer written next iteration must be done
      if (MODE == kModeMain && tid == 0) tma_store_wait_read<1>();
    }
    __syncthreads();
    if (p.use_tma) {
      if (tid == 0) {
        if (MODE == kModeMain) {
          tma_store_3d(&p.tm_y, Ys, d0, t0, b);
          tma_store_commit();
        }
        if (ib + S::NSTAGE < nblk)
          fwd_issue_loads<N, T, MODE>(p, st, &bars[s], d0, t0 + S::NSTAGE * TC, b);
      }
    } else if (MODE == kModeMain) {
      T* y = static_cast<T*>(const_cast<void*>(p.y.ptr));
      for (int e = tid; e < TC * DT; e += Gm::NT) {
        const int tt = e / DT, dd = e % DT;
        const int t = t0 + tt, dg = d0 + dd;
        if (t < p.L && dg < p.D) y[b * p.y.sb + (long long)t * p.y.sl + dg] = Ys[e];
      }
    }
  }

  if (MODE == kModeMain) {
    if (dvalid && t_end == p.L && p.last != nullptr)
      *reinterpret_cast<float4*>(p.last + ((size_t)b * p.D + d) * N + g * 4) = make_float4(h[0], h[1], h[2], h[3]);
  } else if (dvalid) {
    const size_t o = (((size_t)b * p.nseg + seg) * p.D + d) * N + g * 4;
    *reinterpret_cast<float4*>(p.seg_hend + o) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(p.seg_decay + o) = make_float4(P[0], P[1], P[2], P[3]);
  }
  if (MODE == kModeMain && p.use_tma && tid == 0) tma_store_wait_all<0>();
}

// Sequential composition of segment summaries, one thread per (b, d, n):
//   seg_init[s] = carry;  carry = decay[s] * carry + hend[s]
__global__ void ssm_carry_kernel(const CarryParams p);

// Host-side launchers (defined per element type in ssm_fwd_<type>.cu).
template <typename T>
cudaError_t launch_fwd(int N, int method, int mode, const FwdParams& p, dim3 grid, cudaStream_t stream);

}  // namespace ssm
