// ssm_bwd.cuh — backward selective scan on sm_100a.
//
// Replaces kernels/triton_scan.py:143-226 (_bwd_kernel) and :288-319 (the backward driver
// that first re-runs the forward into a (B, L, D_tile, N) HBM buffer `hbuf`), with the math of
// models/scan.py:219-255 (reverse adjoint scan dh_t = g_t + a_{t+1} dh_{t+1}, then gradients
// through discretize).
//
// One CTA owns a (batch, 32-channel tile) and walks the sequence backwards in 16-step chunks.
// For every chunk it (1) TMA-stages u, delta, z, dy and B, C, (2) recomputes the chunk's 16
// states in registers from the checkpoint the forward saved (chunk_states), (3) runs the
// reverse adjoint through those registers.  No per-step state ever touches HBM.
//
// Per element (t, d, n), with dh the total adjoint of h_t (carried + dys_t C_t[n]):
//   q = dh a_t              adjoint flowing to h_{t-1}
//   ddelta_t[d] += sum_n dh dh_t/ddelta,  dA[d,n] += dh dh_t/dA,  du_t[d] += dh dh_t/du
//   dB_t[n] += sum_d dh dh_t/dB,          dC_t[n] += sum_d dys_t[d] h_t[n]
// Reductions over n stay inside a channel group (warp shuffles); reductions over d go
// through a shuffle transposition, a fixed-order cross-warp sum in shared memory and a
// per-CTA partial buffer that ssm_bwd_finalize sums in fixed order: no float atomics, so
// gradients are bitwise reproducible.
//
// ZOH dA uses the identity  A dh_t/dA = delta dh_t/ddelta - coef B u   (coef = expm1(dA)/A),
// so no separate small-z series is needed (the reference evaluates
// f(z) = (z e^z - expm1 z)/z^2 with a series branch, kernels/triton_scan.py:199-202).
#pragma once

#include "ssm_common.cuh"

namespace ssm {

template <int N, typename T>
struct BwdSmem {
  using Gm = Geo<N>;
  static constexpr int NSTAGE = 2;
  static constexpr int NOUT = 2;
  static constexpr int ACT = Gm::TC * Gm::DT * (int)sizeof(T);
  static constexpr int BC = Gm::TC * N * (int)sizeof(T);
  static constexpr int OFF_U = 0, OFF_DT = ACT, OFF_Z = 2 * ACT, OFF_DY = 3 * ACT, OFF_B = 4 * ACT,
                       OFF_C = 4 * ACT + BC;
  static constexpr int STAGE = 4 * ACT + 2 * BC;
  static constexpr int F32T = Gm::TC * Gm::DT * 4;                     // one fp32 (16 x 32) tile
  static constexpr int OFF_DYS = NSTAGE * STAGE;                      // dy * silu(z)
  static constexpr int OFF_SIG = OFF_DYS + F32T;                      // sigmoid(z)
  static constexpr int OFF_OUT = OFF_SIG + F32T;                      // NOUT x {du, ddelta, dz}
  static constexpr int OFF_RED = OFF_OUT + NOUT * 3 * ACT;            // (TC, NW, 2N) fp32
  static constexpr int RED = Gm::TC * Gm::NW * 2 * N * 4;
  static constexpr int OFF_BAR = OFF_RED + RED;
  static constexpr int BYTES = OFF_BAR + NSTAGE * 8;
  static_assert(ACT % 128 == 0 && BC % 128 == 0, "TMA tiles must stay 128-byte aligned");
};

template <int N, typename T>
__device__ __forceinline__ void bwd_issue_loads(const BwdParams& p, unsigned char* st, uint64_t* bar, int d0,
                                                int t0, int b) {
  using S = BwdSmem<N, T>;
  const uint32_t tx = 3 * S::ACT + 2 * S::BC + (p.has_z ? S::ACT : 0);
  mbar_arrive_expect_tx(bar, tx);
  tma_load_3d(st + S::OFF_U, &p.tm_u, bar, d0, t0, b);
  tma_load_3d(st + S::OFF_DT, &p.tm_dt, bar, d0, t0, b);
  tma_load_3d(st + S::OFF_DY, &p.tm_dy, bar, d0, t0, b);
  tma_load_3d(st + S::OFF_B, &p.tm_B, bar, 0, t0, b);
  tma_load_3d(st + S::OFF_C, &p.tm_C, bar, 0, t0, b);
  if (p.has_z) tma_load_3d(st + S::OFF_Z, &p.tm_z, bar, d0, t0, b);
}

template <int N, typename T>
__device__ __forceinline__ void bwd_coop_load(const BwdParams& p, unsigned char* st, int d0, int t0, int b) {
  using Gm = Geo<N>;
  using S = BwdSmem<N, T>;
  const T zero = from_f32<T>(0.0f);
  for (int e = threadIdx.x; e < Gm::TC * Gm::DT; e += Gm::NT) {
    const int tt = e / Gm::DT, dd = e % Gm::DT;
    const int t = t0 + tt, dg = d0 + dd;
    const bool ok = t < p.L && dg < p.D;
    const long long tl = t;
    reinterpret_cast<T*>(st + S::OFF_U)[e] =
        ok ? static_cast<const T*>(p.u.ptr)[b * p.u.sb + tl * p.u.sl + dg] : zero;
    reinterpret_cast<T*>(st + S::OFF_DT)[e] =
        ok ? static_cast<const T*>(p.dt.ptr)[b * p.dt.sb + tl * p.dt.sl + dg] : zero;
    reinterpret_cast<T*>(st + S::OFF_DY)[e] =
        ok ? static_cast<const T*>(p.dy.ptr)[b * p.dy.sb + tl * p.dy.sl + dg] : zero;
    if (p.has_z)
      reinterpret_cast<T*>(st + S::OFF_Z)[e] =
          ok ? static_cast<const T*>(p.z.ptr)[b * p.z.sb + tl * p.z.sl + dg] : zero;
  }
  for (int e = threadIdx.x; e < Gm::TC * N; e += Gm::NT) {
    const int tt = e / N, n = e % N;
    const int t = t0 + tt;
    const bool ok = t < p.L;
    reinterpret_cast<T*>(st + S::OFF_B)[e] =
        ok ? static_cast<const T*>(p.Bm.ptr)[b * p.Bm.sb + (long long)t * p.Bm.sl + n] : zero;
    reinterpret_cast<T*>(st + S::OFF_C)[e] =
        ok ? static_cast<const T*>(p.Cm.ptr)[b * p.Cm.sb + (long long)t * p.Cm.sl + n] : zero;
  }
}

template <int N, int METHOD, typename T>
__global__ void __launch_bounds__(Geo<N>::NT) ssm_bwd_kernel(const __grid_constant__ BwdParams p) {
  using Gm = Geo<N>;
  using S = BwdSmem<N, T>;
  constexpr int TC = Gm::TC, DT = Gm::DT, LPC = Gm::LPC, CPW = Gm::CPW, NW = Gm::NW;
  constexpr int TG = (LPC <= 4) ? LPC : 1;          // time steps per (y, du, ddelta) reduction
  constexpr int RV = 4 * TG;                         // values per reduction (y, du, ddelta, pad)
  constexpr int VPL = (8 >= CPW) ? 8 / CPW : 1;      // dB|dC values per lane after transposition
  constexpr int DUP = (CPW > 8) ? CPW / 8 : 1;       // lanes holding the same dB|dC value
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  float* SDYS = reinterpret_cast<float*>(smem + S::OFF_DYS);
  float* SSIG = reinterpret_cast<float*>(smem + S::OFF_SIG);
  float* SRED = reinterpret_cast<float*>(smem + S::OFF_RED);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = lane / LPC, g = lane % LPC;
  const int dl = warp * CPW + c;
  const int b = blockIdx.y, dtile = blockIdx.x;
  const int d0 = dtile * DT, d = d0 + dl;
  const bool dvalid = d < p.D;
  const int nch = p.nchunks;

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
  const float Dd = (p.Dskip != nullptr && dvalid) ? p.Dskip[d] : 0.0f;
  const size_t bd = ((size_t)b * p.D + d) * N + g * 4;

  float dh[4] = {0.f, 0.f, 0.f, 0.f};
  if (dvalid && p.dlast != nullptr) load4(p.dlast + bd, dh);
  float dAA[4] = {0.f, 0.f, 0.f, 0.f};
  float dDacc = 0.0f;

  if (p.use_tma) {
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < S::NSTAGE; ++s) mbar_init(&bars[s], 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
      for (int s = 0; s < S::NSTAGE && s < nch; ++s)
        bwd_issue_loads<N, T>(p, smem + s * S::STAGE, &bars[s], d0, (nch - 1 - s) * TC, b);
    }
  }

  auto cs_ptr = [&](int ch) { return p.chunk_states + (((size_t)b * nch + ch) * p.D + d) * N + g * 4; };
  float hs[4] = {0.f, 0.f, 0.f, 0.f};
  if (dvalid) load4(cs_ptr(nch - 1), hs);

  for (int i = 0; i < nch; ++i) {
    const int ch = nch - 1 - i;
    const int s = i % S::NSTAGE;
    const int t0 = ch * TC;
    unsigned char* st = smem + s * S::STAGE;
    float hs_next[4] = {0.f, 0.f, 0.f, 0.f};
    if (dvalid && ch > 0) load4(cs_ptr(ch - 1), hs_next);

    if (p.use_tma) {
      mbar_wait(&bars[s], (uint32_t)((i / S::NSTAGE) & 1), p.err);
    } else {
      bwd_coop_load<N, T>(p, st, d0, t0, b);
      __syncthreads();
    }
    const T* Xs = reinterpret_cast<const T*>(st + S::OFF_U);
    const T* DLs = reinterpret_cast<const T*>(st + S::OFF_DT);
    const T* Zs = reinterpret_cast<const T*>(st + S::OFF_Z);
    const T* DYs = reinterpret_cast<const T*>(st + S::OFF_DY);
    const T* Bs = reinterpret_cast<const T*>(st + S::OFF_B);
    const T* Cs = reinterpret_cast<const T*>(st + S::OFF_C);

    // Gate terms once per (t, d):  dys = dy * silu(z)  (the scan's output gradient)
    for (int e = tid; e < TC * DT; e += Gm::NT) {
      const float dyv = to_f32(DYs[e]);
      if (p.has_z) {
        const float zz = to_f32(Zs[e]);
        const float sg = sigmoid(zz);
        SSIG[e] = sg;
        SDYS[e] = dyv * zz * sg;
      } else {
        SDYS[e] = dyv;
      }
    }
    __syncthreads();

    // (2) recompute the chunk's states from its checkpoint
    float H[TC][4];
    {
      float hc[4] = {hs[0], hs[1], hs[2], hs[3]};
#pragma unroll
      for (int j = 0; j < TC; ++j) {
        const float uu = to_f32(Xs[j * DT + dl]);
        const float dtv = to_f32(DLs[j * DT + dl]);
        const float dtu = dtv * uu;
        float Bn[4];
        load4(Bs + j * N + g * 4, Bn);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (METHOD == kZOH) {
            const float a = ex2(dtv * A2[k]);
            const float gg = (Bn[k] * uu) * iA[k];
            hc[k] = fmaf(a, hc[k] + gg, -gg);
          } else if (METHOD == kEuler) {
            hc[k] = fmaf(ex2(dtv * A2[k]), hc[k], dtu * Bn[k]);
          } else {
            const float zz = dtv * Ak[k];
            const float w = rcp(fmaf(-0.5f, zz, 1.0f));
            hc[k] = fmaf(fmaf(0.5f, zz, 1.0f) * w, hc[k], (dtu * Bn[k]) * w);
          }
          H[j][k] = hc[k];
        }
      }
    }

    // (3) reverse adjoint through the chunk
    T* DUo = reinterpret_cast<T*>(smem + S::OFF_OUT + (i % S::NOUT) * 3 * S::ACT);
    T* DDTo = DUo + TC * DT;
    T* DZo = DDTo + TC * DT;
#pragma unroll
    for (int jg = TC / TG - 1; jg >= 0; --jg) {
      float red[RV];
#pragma unroll
      for (int jj = TG - 1; jj >= 0; --jj) {
        const int j = jg * TG + jj;
        const float uu = to_f32(Xs[j * DT + dl]);
        const float dtv = to_f32(DLs[j * DT + dl]);
        const float dys = SDYS[j * DT + dl];
        float Bn[4], Cn[4];
        load4(Bs + j * N + g * 4, Bn);
        load4(Cs + j * N + g * 4, Cn);
        float yv = 0.f, duv = 0.f, ddtv = 0.f;
        float bc[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float ht = H[j][k];
          const float hp = (j > 0) ? H[j > 0 ? j - 1 : 0][k] : hs[k];
          const float Bu = Bn[k] * uu;
          dh[k] = fmaf(dys, Cn[k], dh[k]);
          bc[4 + k] = dys * ht;
          yv = fmaf(Cn[k], ht, yv);
          if (METHOD == kZOH) {
            const float a = ex2(dtv * A2[k]);
            const float q = dh[k] * a;
            const float sv = q * fmaf(Ak[k], hp, Bu);
            ddtv += sv;
            const float pp = (q - dh[k]) * iA[k];
            duv = fmaf(pp, Bn[k], duv);
            bc[k] = pp * uu;
            dAA[k] = fmaf(dtv, sv, dAA[k]);
            dAA[k] = fmaf(-pp, Bu, dAA[k]);
            dh[k] = q;
          } else if (METHOD == kEuler) {
            const float a = ex2(dtv * A2[k]);
            const float q = dh[k] * a;
            const float sv = fmaf(q * Ak[k], hp, dh[k] * Bu);
            ddtv += sv;
            const float pp = dh[k] * dtv;
            duv = fmaf(pp, Bn[k], duv);
            bc[k] = pp * uu;
            dAA[k] = fmaf(dtv * q, hp, dAA[k]);
            dh[k] = q;
          } else {
            const float zz = dtv * Ak[k];
            const float w = rcp(fmaf(-0.5f, zz, 1.0f));
            const float a = fmaf(0.5f, zz, 1.0f) * w;
            const float dhw2 = dh[k] * w * w;
            const float sv = dhw2 * fmaf(Ak[k], hp, Bu);
            ddtv += sv;
            const float pp = dh[k] * dtv * w;
            duv = fmaf(pp, Bn[k], duv);
            bc[k] = pp * uu;
            dAA[k] = fmaf(dtv * dhw2, fmaf(0.5f * dtv, Bu, hp), dAA[k]);
            dh[k] = dh[k] * a;
          }
        }
        // dB | dC: sum over this warp's channels, then park per (t, warp) for the cross-warp sum
        xpose_reduce<8, CPW, LPC>(bc, lane);
        if (c % DUP == 0) {
#pragma unroll
          for (int v = 0; v < VPL; ++v) {
            const int idx = (c / DUP) * VPL + v;   // quantity: (idx >> 2) = 0 dB / 1 dC, state g*4 + (idx & 3)
            SRED[(j * NW + warp) * 2 * N + (idx >> 2) * N + g * 4 + (idx & 3)] = bc[v];
          }
        }
        red[jj * 4 + 0] = yv;
        red[jj * 4 + 1] = duv;
        red[jj * 4 + 2] = ddtv;
        red[jj * 4 + 3] = 0.f;
      }
      // (y, du, ddelta) over the LPC lanes of the channel
      float yv, duv, ddtv;
      int j;
      if (TG == LPC) {
        xpose_reduce<RV, LPC, 1>(red, lane);  // lane g: timestep jg*TG + g
        yv = red[0]; duv = red[1]; ddtv = red[2];
        j = jg * TG + g;
      } else {                                 // TG == 1, LPC > 4
        yv = group_allreduce<LPC, 1>(red[0]);
        duv = group_allreduce<LPC, 1>(red[1]);
        ddtv = group_allreduce<LPC, 1>(red[2]);
        j = jg;
      }
      if (TG == LPC || g == 0) {
        const float uu = to_f32(Xs[j * DT + dl]);
        const float dys = SDYS[j * DT + dl];
        DUo[j * DT + dl] = from_f32<T>(duv + Dd * dys);
        DDTo[j * DT + dl] = from_f32<T>(ddtv);
        if (p.has_z) {
          const float zz = to_f32(Zs[j * DT + dl]);
          const float sg = SSIG[j * DT + dl];
          const float dyv = to_f32(DYs[j * DT + dl]);
          const float yfull = fmaf(Dd, uu, yv);
          DZo[j * DT + dl] = from_f32<T>(dyv * yfull * sg * fmaf(zz, 1.0f - sg, 1.0f));
        }
        dDacc = fmaf(dys, uu, dDacc);
      }
    }

    if (p.use_tma) {
      fence_proxy_async_smem();
    }
    __syncthreads();

    // cross-warp dB | dC sum -> this CTA's partial (fixed order)
    for (int e = tid; e < TC * 2 * N; e += Gm::NT) {
      const int j = e / (2 * N), v = e % (2 * N);
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) sum += SRED[(j * NW + w) * 2 * N + v];
      const int t = t0 + j;
      if (t < p.L) p.part_bc[(((size_t)b * p.ndt + dtile) * p.L + t) * 2 * N + v] = sum;
    }

    if (p.use_tma) {
      if (tid == 0) {
        tma_store_3d(&p.tm_du, DUo, d0, t0, b);
        tma_store_3d(&p.tm_ddt, DDTo, d0, t0, b);
        if (p.has_z) tma_store_3d(&p.tm_dz, DZo, d0, t0, b);
        tma_store_commit();
        if (ch - S::NSTAGE >= 0) bwd_issue_loads<N, T>(p, st, &bars[s], d0, (ch - S::NSTAGE) * TC, b);
        // the output buffer written next chunk was last read by the store issued one chunk ago
        tma_store_wait_read<1>();
      }
    } else {
      for (int e = tid; e < TC * DT; e += Gm::NT) {
        const int tt = e / DT, dd = e % DT;
        const int t = t0 + tt, dg = d0 + dd;
        if (t < p.L && dg < p.D) {
          const long long tl = t;
          static_cast<T*>(const_cast<void*>(p.du.ptr))[b * p.du.sb + tl * p.du.sl + dg] = DUo[e];
          static_cast<T*>(const_cast<void*>(p.ddt.ptr))[b * p.ddt.sb + tl * p.ddt.sl + dg] = DDTo[e];
          if (p.has_z) static_cast<T*>(const_cast<void*>(p.dz.ptr))[b * p.dz.sb + tl * p.dz.sl + dg] = DZo[e];
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) hs[k] = hs_next[k];
  }

  // per-(b, d) partials; ssm_bwd_finalize sums them over b in fixed order
  dDacc = group_allreduce<LPC, 1>(dDacc);
  if (dvalid) {
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = (METHOD == kZOH) ? dAA[k] * iA[k] : dAA[k];
    *reinterpret_cast<float4*>(p.part_A + bd) = make_float4(o[0], o[1], o[2], o[3]);
    if (p.dh0 != nullptr) *reinterpret_cast<float4*>(p.dh0 + bd) = make_float4(dh[0], dh[1], dh[2], dh[3]);
    if (g == 0) p.part_D[(size_t)b * p.D + d] = dDacc;
  }
  if (p.use_tma && tid == 0) tma_store_wait_all<0>();
}

// Sums the per-CTA dB | dC partials over channel tiles and the dA / dD partials over batch,
// each in a fixed order, and writes dB, dC (element type T), dA, dD (fp32).
template <typename T>
__global__ void ssm_bwd_finalize(const FinParams p) {
  const long long n2 = 2LL * p.N;
  const long long nbc = (long long)p.B * p.L * n2;
  const long long nA = (long long)p.D * p.N;
  const long long total = nbc + nA + (p.dD != nullptr ? p.D : 0);
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    if (idx < nbc) {
      const int v = (int)(idx % n2);
      const long long bt = idx / n2;
      const int t = (int)(bt % p.L), b = (int)(bt / p.L);
      float s = 0.f;
      for (int q = 0; q < p.ndt; ++q) s += p.part_bc[(((size_t)b * p.ndt + q) * p.L + t) * n2 + v];
      if (v < p.N) {
        static_cast<T*>(const_cast<void*>(p.dB.ptr))[b * p.dB.sb + (long long)t * p.dB.sl + v] = from_f32<T>(s);
      } else {
        static_cast<T*>(const_cast<void*>(p.dC.ptr))[b * p.dC.sb + (long long)t * p.dC.sl + (v - p.N)] =
            from_f32<T>(s);
      }
    } else if (idx < nbc + nA) {
      const long long i = idx - nbc;
      float s = 0.f;
      for (int b = 0; b < p.B; ++b) s += p.part_A[(size_t)b * nA + i];
      p.dA[i] = s;
    } else {
      const long long dd = idx - nbc - nA;
      float s = 0.f;
      for (int b = 0; b < p.B; ++b) s += p.part_D[(size_t)b * p.D + dd];
      p.dD[dd] = s;
    }
  }
}

template <typename T>
cudaError_t launch_bwd(int N, int method, const BwdParams& p, dim3 grid, cudaStream_t stream);
template <typename T>
cudaError_t launch_bwd_finalize(const FinParams& p, cudaStream_t stream);

}  // namespace ssm
