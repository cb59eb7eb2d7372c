// ssm_bwd.cuh — backward selective scan on sm_100a.
//
// Replaces kernels/triton_scan.py:143-226 (_bwd_kernel) and :288-319 (the backward driver
// that first re-runs the forward into a (B, L, D_tile, N) HBM buffer `hbuf`), with the math of
// models/scan.py:219-255 (reverse adjoint scan dh_t = g_t + a_{t+1} dh_{t+1}, then gradients
// through discretize).
//
// One CTA owns a (batch, 32-channel tile, sequence segment) and walks its segment backwards in
// 16-step chunks.  Grids with fewer CTAs than the GPU holds at once (long sequences over few
// channels) split the sequence into segments: each starts from the adjoint entering it from the
// right, which the adjoint summaries of the later segments give (the forward kernel's adjoint mode
// and the reverse carry; one segment takes dlast).
// For every chunk it
//   (1) TMA-stages u, delta, z, dy, the saved pre-gate output and B, C;
//   (2) gate pass, once per (t, d): dys = dy silu(z), dz (stored straight to global memory), dD,
//       the step size (activated when dt_softplus), packed with u as one float4 per (t, d); and G
//       state-permuted fp32 copies of the B, C tiles (see "state permutation" below);
//   (3) recomputes the chunk's 16 states in registers from the checkpoint the forward saved
//       (chunk_states), and keeps each step's discretisation coefficient -- the one MUFU-derived
//       value the reverse pass needs (ZOH: r = A rho = expm1(delta A) - delta A, Euler: a, bilinear:
//       1 / (1 - delta A / 2)) -- in a thread-private shared-memory slot;
//   (4) runs the reverse adjoint through those registers, reading the coefficients back instead
//       of re-evaluating exponentials (ZOH: coef = delta + r / A, a = 1 + A coef); the bf16 N = 16
//       layout keeps no cache and re-evaluates them, which fits a third CTA on every SM.
// Both passes fetch step j+-1's inputs while step j computes, and step j's dB|dC reduction is
// issued after step j-1's arithmetic, so shared-memory and shuffle latency overlap work.
// du and ddelta go through padded shared tiles (two sets, stored coalesced at the end of each
// chunk); dz leaves straight from the gate pass (a warp writes one 32-channel row).  No per-step
// state ever touches HBM.
//
// Per element (t, d, n), with dh the total adjoint of h_t (carried + dys_t C_t[n]):
//   q = dh a_t                      adjoint flowing to h_{t-1}
//   ddelta_t[d] += sum_n dh dh_t/ddelta,   du_t[d] += sum_n dh dh_t/du,   dA[d,n] += dh dh_t/dA,
//   dB_t[n] += sum_d dh dh_t/dB,           dC_t[n] += sum_d dys_t[d] h_t[n]
// ZOH.  coef = expm1(z) / A (z = delta A) enters through rho = coef - delta = (expm1(z) - z) / A,
// evaluated without cancellation (zoh_r below).  With a = 1 + A coef and h_t = a h_{t-1} + coef B u,
//   A dh_t/dA = z a h_{t-1} + B u (delta a - coef) = z h_t - rho B u,
// an exact identity (delta a - coef = z coef - rho) whose two terms do not cancel: the B u parts of
// z h_t and rho B u stand about 2 : 1 for small z.  So dA = (sum_t dh_t (z h_t - rho B u)) / A costs
// two FMAs per element and stays accurate in relative terms for every z and every A, where the
// reference evaluates f(z) = (z e^z - expm1 z) / z^2 with a series branch
// (kernels/triton_scan.py:199-202) and forming A dA as delta dh/ddelta - coef B u would lose about
// 1e-7 / |A| relative (1e-2 at |A| = 1e-3 in the transient of small steps).  In the reverse pass the
// two sums are kept apart, dA = sum dh delta h_t - (1/A^2) sum (dh r) B u with r = A rho (what the
// recompute pass caches), and their products dh delta and dh r also give pc = dh coef = dh delta +
// (dh r) / A and q = dh a = dh + A pc: six packed operations per state pair for q, pc and dA.
// The step-size term uses the same identity: dh_t/ddelta = A a h_{t-1} + a B u = A h_t + B u (ZOH).
//
// Reductions: over n inside a channel's lane group (shuffle transposition); over d by a
// shuffle transposition across the warp's channels, a fixed-order cross-warp sum in shared
// memory and a per-CTA partial that ssm_bwd_finalize sums in fixed order.  No float atomics:
// gradients are bitwise reproducible.
//
// State permutation: lane c of a channel group keeps its G states in register slots
// j -> state G g + (j ^ perm(c)), perm taken from the log2(G) highest bits of c.  Then the
// first log2(G) halving stages of the dB|dC transposition send a fixed register slot on every
// lane (no lane-dependent selects).  The B, C tiles are staged as G copies, one per perm, so
// every lane still reads its G values with one vector shared load.
#pragma once

#include "ssm_common.cuh"

namespace ssm {

template <int N, int G, typename T>
struct BwdSmem {
  using Gm = Geo<N, G>;
  static constexpr int TC = Gm::TC, DT = Gm::DT;
  static constexpr int NSTAGE = 2;
  // bf16 at N = 16 trades the coefficient cache for a third CTA per SM (168 registers, no cache:
  // the reverse pass re-evaluates the coefficients).  With the large grids of bf16 layers (config
  // 3: 1280 CTAs) the extra warps win: 9.53 -> 9.21 ms per backward at config 3, one B200.  fp32
  // at config 1 (256 CTAs, under two per SM) keeps the cache.
  static constexpr bool TRIO = N == 16 && G == 4 && sizeof(T) == 2;
  static constexpr int ACT = TC * DT * (int)sizeof(T);
  static constexpr int BC = TC * N * (int)sizeof(T);
  static constexpr int OFF_U = 0, OFF_DT = ACT, OFF_Z = 2 * ACT, OFF_DY = 3 * ACT, OFF_YG = 4 * ACT,
                       OFF_B = 5 * ACT, OFF_C = 5 * ACT + BC;
  static constexpr int STAGE = 5 * ACT + 2 * BC;
  // Gate-pass products of one chunk: per (t, d) {u, delta (activated when dt_softplus), dy silu(z),
  // sigmoid(raw delta + bias) (dt_softplus)}, packed for one 128-bit load per step, and the G
  // state-permuted fp32 copies of B and C.
  static constexpr int SUDB = TC * DT * 16;
  // one perm copy of a (16 x N) tile, padded by 16 floats: a warp's lanes read G-vectors at G
  // perms x LPC groups; with copies 1 KB apart all perms hit the same banks (a G-way conflict),
  // with 64 extra bytes consecutive perms land half a bank row apart (2-way, the minimum for 16
  // distinct 16-byte vectors)
  static constexpr int PCP = TC * N + 16;                     // perm copy pitch (floats)
  static constexpr int BPB = G * PCP * 4;
  // du and ddelta tiles, read or written in (step, channel) blocks of the lane layout: a padded
  // row pitch spreads such a block over the 32 banks; two sets (chunk i and i + 1)
  static constexpr int OP = PadPitch<Gm::CPW, T>::value;
  static constexpr int OUT = ((TC * OP * (int)sizeof(T)) + 127) / 128 * 128;
  static constexpr int NOUT = 2;
  // the recompute pass's per-step coefficients: TC steps x NT threads x G values (thread-private);
  // layouts where they do not fit (N = 64: 128 KB), and the three-CTA layout, re-evaluate them in
  // the reverse pass instead
  static constexpr int CFB_FULL = TC * Gm::NT * G * 4;
  static constexpr int BASE = NSTAGE * STAGE + TC * Gm::NW * 2 * N * 4 + Gm::NT * 4 + NSTAGE * 8 + NOUT * 2 * OUT;
  static constexpr bool CACHE = !TRIO && BASE + CFB_FULL + SUDB + 2 * BPB <= 227 * 1024;
  static constexpr int CFB = CACHE ? CFB_FULL : 0;
  static constexpr int FIXED = BASE + CFB;
  // bytes with gate products GA chunks ahead: GA + 1 product buffers
  static constexpr int bytes_for(int ga) { return FIXED + (ga + 1) * (SUDB + 2 * BPB); }
  // per-CTA budget that keeps the CTAs per SM the register file allows (256 threads' worth of
  // registers at most per 128 threads, G = 2 launches capped at two CTAs per SM, the three-CTA
  // layout at three)
  static constexpr int CTAS = TRIO ? 3 : (G == 2 || Gm::NT >= 256) ? (G == 2 ? 2 : 1) : 256 / Gm::NT;
  static constexpr int MINB = TRIO ? 3 : (G == 2 ? 2 : 1);   // the kernel's register cap
  static constexpr int BUDGET = 228 * 1024 / CTAS - 1024 < 227 * 1024 ? 228 * 1024 / CTAS - 1024 : 227 * 1024;
  // GA = 1: chunk i + 1's gate pass runs inside chunk i's reverse pass, so the gate products are
  // double-buffered; layouts that would lose a CTA per SM that way keep one gate buffer (GA = 0)
  // and run the gate pass at the top of its own chunk.
  static constexpr int GA = bytes_for(1) <= BUDGET ? 1 : 0;
  static constexpr int NBUF = GA + 1;          // gate-product buffers
  static constexpr int OFF_SUD = NSTAGE * STAGE;
  static constexpr int OFF_BP = OFF_SUD + NBUF * SUDB;          // NBUF x G perms x (16 x N) fp32 B
  static constexpr int OFF_CP = OFF_BP + NBUF * BPB;            // NBUF x G perms x (16 x N) fp32 C
  static constexpr int OFF_CF = OFF_CP + NBUF * BPB;            // (TC, NT, G) fp32 coefficients
  static constexpr int OFF_OUT = OFF_CF + CFB;                  // NOUT x {du, ddelta} tiles
  static constexpr int OFF_RED = OFF_OUT + NOUT * 2 * OUT;      // (TC, NW, 2N) fp32
  static constexpr int OFF_DD = OFF_RED + TC * Gm::NW * 2 * N * 4;   // NT floats (dD partials)
  static constexpr int OFF_BAR = OFF_DD + Gm::NT * 4;
  static constexpr int BYTES = OFF_BAR + NSTAGE * 8;
  static_assert(ACT % 128 == 0 && BC % 128 == 0, "TMA tiles must stay 128-byte aligned");
  static_assert(OFF_CF % 16 == 0, "coefficient slots must stay 16-byte aligned");
  static_assert(N != 16 || G != 4 || CACHE || TRIO, "the fp32 N = 16 layout keeps its coefficients");
  static_assert(!TRIO || BYTES <= BUDGET, "the three-CTA layout must fit three CTAs per SM");
  static_assert(BYTES <= 227 * 1024, "backward shared-memory layout exceeds a CTA's limit");
};

template <typename S>
__device__ __forceinline__ void bwd_issue_loads(const BwdParams& p, unsigned char* st, uint64_t* bar, int d0,
                                                int t0, int b) {
  const uint32_t tx = 3 * S::ACT + 2 * S::BC + (p.has_z ? 2 * S::ACT : 0);
  mbar_arrive_expect_tx(bar, tx);
  tma_load_3d(st + S::OFF_U, &p.tm_u, bar, d0, t0, b);
  tma_load_3d(st + S::OFF_DT, &p.tm_dt, bar, d0, t0, b);
  tma_load_3d(st + S::OFF_DY, &p.tm_dy, bar, d0, t0, b);
  tma_load_3d(st + S::OFF_B, &p.tm_B, bar, 0, t0, b);
  tma_load_3d(st + S::OFF_C, &p.tm_C, bar, 0, t0, b);
  if (p.has_z) {
    tma_load_3d(st + S::OFF_Z, &p.tm_z, bar, d0, t0, b);
    tma_load_3d(st + S::OFF_YG, &p.tm_yg, bar, d0, t0, b);
  }
}

template <typename S, int N, int NT, typename T>
__device__ __forceinline__ void bwd_coop_load(const BwdParams& p, unsigned char* st, int d0, int t0, int b) {
  const T zero = from_f32<T>(0.0f);
  for (int e = threadIdx.x; e < S::TC * S::DT; e += NT) {
    const int tt = e / S::DT, dd = e % S::DT;
    const int t = t0 + tt, dg = d0 + dd;
    const bool ok = t < p.L && dg < p.D;
    const long long tl = t;
    auto ld = [&](const DAct& a) { return ok ? static_cast<const T*>(a.ptr)[b * a.sb + tl * a.sl + dg] : zero; };
    reinterpret_cast<T*>(st + S::OFF_U)[e] = ld(p.u);
    reinterpret_cast<T*>(st + S::OFF_DT)[e] = ld(p.dt);
    reinterpret_cast<T*>(st + S::OFF_DY)[e] = ld(p.dy);
    if (p.has_z) {
      reinterpret_cast<T*>(st + S::OFF_Z)[e] = ld(p.z);
      reinterpret_cast<T*>(st + S::OFF_YG)[e] = ld(p.yg);
    }
  }
  for (int e = threadIdx.x; e < S::TC * N; e += NT) {
    const int tt = e / N, n = e % N;
    const int t = t0 + tt;
    const bool ok = t < p.L;
    reinterpret_cast<T*>(st + S::OFF_B)[e] =
        ok ? static_cast<const T*>(p.Bm.ptr)[b * p.Bm.sb + (long long)t * p.Bm.sl + n] : zero;
    reinterpret_cast<T*>(st + S::OFF_C)[e] =
        ok ? static_cast<const T*>(p.Cm.ptr)[b * p.Cm.sb + (long long)t * p.Cm.sl + n] : zero;
  }
}

constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v / 2); }

// ZOH's r = expm1(z) - z = A rho (z = delta A, x = z log2 e) for a pair, given a = ex2(x): A times the
// part of the input coefficient beyond its leading term, rho = coef - delta = (expm1(z) - z) / A,
// evaluated without cancellation (the 1/A is applied where r is used: coef = delta + r / A).  Both
// candidates are lower bounds of r for every z (as in em1x2):
// the polynomial z^2/2 + z^3/6 (its remainder e^xi z^4/24 is >= 0) and the biased MUFU value
// minus z; their maximum is within min(z^4/24, 3.9e-7 e^z) of r.  Relative to coef = delta + rho
// that is the error bound of em1x2 (7e-6 at most); relative to rho itself (about delta z / 2) it is
// z^2/12 below |z| = 0.055 and 7.8e-7 / z^2 above, 2.6e-4 at most (the rho B u term of dA).
__device__ __forceinline__ float2 zoh_r(float2 x, float2 a) {
  const float2 e = fma2(a, bc2(kEm1Scale), bc2(-1.0f));
  const float2 rp = mul2(mul2(x, x), fma2(x, bc2(kEm1C3), bc2(kEm1C2)));
  const float2 rm = fma2(x, bc2(-kLn2), e);
  return make_float2(fmaxf(rp.x, rm.x), fmaxf(rp.y, rm.y));
}

// G = 2 exists to raise occupancy, so its register budget is capped at two CTAs per SM; the bf16
// N = 16 layout is capped at three.
template <int N, int G, int METHOD, typename T>
__global__ void __launch_bounds__(Geo<N, G>::NT, BwdSmem<N, G, T>::MINB) ssm_bwd_kernel(const __grid_constant__ BwdParams p) {
  using Gm = Geo<N, G>;
  using S = BwdSmem<N, G, T>;
  constexpr int TC = Gm::TC, DT = Gm::DT, LPC = Gm::LPC, CPW = Gm::CPW, NW = Gm::NW, NT = Gm::NT;
  constexpr int NP = G / 2;                            // state pairs per thread
  constexpr int LC = ilog2(CPW), LG = ilog2(G);
  constexpr int NSLOT = LC < LG ? LC : LG;             // slot-splitting stages (select-free)
  constexpr bool QSTAGE = LC > LG;                     // a dB / dC splitting stage follows
  constexpr int BCPL = QSTAGE ? 1 : (LC == LG ? 2 : 4);   // dB|dC values per lane at the end
  constexpr int BCDUP = (LC > LG + 1) ? (1 << (LC - LG - 1)) : 1;
  // (du, ddelta) over the LPC lanes of a channel, 4 steps per transposition: V = 8 values
  constexpr int QV = 8;
  constexpr int QPL = (QV >= LPC) ? QV / LPC : 1;      // values per lane afterwards
  constexpr int QDUP = (LPC > QV) ? LPC / QV : 1;      // lanes holding the same value
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  float4* __restrict__ SUD = reinterpret_cast<float4*>(smem + S::OFF_SUD);
  float* __restrict__ SBP = reinterpret_cast<float*>(smem + S::OFF_BP);
  float* __restrict__ SCP = reinterpret_cast<float*>(smem + S::OFF_CP);
  float* __restrict__ SCF = reinterpret_cast<float*>(smem + S::OFF_CF);
  float* __restrict__ SRED = reinterpret_cast<float*>(smem + S::OFF_RED);
  float* __restrict__ SDD = reinterpret_cast<float*>(smem + S::OFF_DD);
  pdl_launch_dependents();
  pdl_wait();

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = lane / LPC, g = lane % LPC;
  const int dl = warp * CPW + c;
  const int b = blockIdx.y, dtile = blockIdx.x;
  const int d0 = dtile * DT, d = d0 + dl;
  const bool dvalid = d < p.D;
  // the CTA's sequence segment (blockIdx.z): chunks [ctop - nch + 1, ctop], walked from ctop down
  const int seg = blockIdx.z;
  const int c_first = seg * (p.seg_len / TC);
  const int ctop = min(p.nchunks, c_first + p.seg_len / TC) - 1;
  const int nch = ctop + 1 - c_first;
  const int nbase = g * G;
  // register slot j holds state nbase + (j ^ perm); slot bit (LG-1-s) = c bit (LC-1-s)
  int perm = 0;
#pragma unroll
  for (int s2 = 0; s2 < NSLOT; ++s2) perm |= ((c >> (LC - 1 - s2)) & 1) << (LG - 1 - s2);

  auto slot_load = [&](const float* src, float2 (&o)[NP]) {   // G values at src, slot order
#pragma unroll
    for (int i = 0; i < NP; ++i)
      o[i] = dvalid ? make_float2(src[(2 * i) ^ perm], src[(2 * i + 1) ^ perm]) : bc2(0.f);
  };
  float2 Ak[NP], A2[NP], iA[NP];
  {
    float2 av[NP];
    slot_load(p.A + (size_t)d * N + nbase, av);
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      if (!dvalid) av[i] = bc2(-1.f);
      Ak[i] = av[i];
      A2[i] = mul2(av[i], bc2(kLog2e));
      iA[i] = make_float2(1.0f / av[i].x, 1.0f / av[i].y);
    }
  }
  const float Dd = (p.Dskip != nullptr && dvalid) ? p.Dskip[d] : 0.0f;
  const size_t bd = ((size_t)b * p.D + d) * N + nbase;
  const size_t bsd = (size_t)b * p.nseg + seg;            // (batch, segment) partial group
  const size_t pbd = (bsd * p.D + d) * N + nbase;

  float2 dh[NP], dAA[NP], dAR[NP];
  // the adjoint entering the segment from its right: dlast for the last segment, else the composed
  // adjoint summaries of the segments after it
  const float* const dh_in = (seg == p.nseg - 1) ? (p.dlast != nullptr ? p.dlast + bd : nullptr) : p.seg_dh + pbd;
  if (dh_in != nullptr) {
    slot_load(dh_in, dh);
  } else {
#pragma unroll
    for (int i = 0; i < NP; ++i) dh[i] = bc2(0.f);
  }
#pragma unroll
  for (int i = 0; i < NP; ++i) dAA[i] = dAR[i] = bc2(0.f);
  float dDacc = 0.0f;
  float dtbacc = 0.0f;         // this thread's share of d loss / d dt_bias for channel dl
  // the gate pass visits elements e = tid + k NT, always channel d0 + tid % DT
  const float dtb_gate = (p.dt_softplus && p.dt_bias != nullptr && d0 + tid % DT < p.D) ? p.dt_bias[d0 + tid % DT] : 0.f;

  if (p.use_tma) {
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < S::NSTAGE; ++s) mbar_init(&bars[s], 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
      for (int s = 0; s < S::NSTAGE && s < nch; ++s)
        bwd_issue_loads<S>(p, smem + s * S::STAGE, &bars[s], d0, (ctop - s) * TC, b);
    }
  }

  // Chunk ci (loop order: ci = 0 is the last chunk of the sequence) lives in stage ci % NSTAGE;
  // acquire(ci) returns once its input tiles are in shared memory.
  auto acquire = [&](int ci) {
    if (p.use_tma) {
      mbar_wait(&bars[ci % S::NSTAGE], (uint32_t)((ci / S::NSTAGE) & 1), p.err);
    } else {
      bwd_coop_load<S, N, NT, T>(p, smem + (ci % S::NSTAGE) * S::STAGE, d0, (ctop - ci) * TC, b);
      __syncthreads();
    }
  };
  T* const dz_out = static_cast<T*>(const_cast<void*>(p.dz.ptr)) + b * p.dz.sb;
  // (2) gate pass over the (t, d) tile of chunk ci: element e = tid + k NT.  Writes the packed
  // per-(t, d) inputs of the recompute and reverse passes, stores dz, and adds the element's d(D)
  // term (only when `live`: a pass over a chunk past the end is discarded).
  constexpr int NE = TC * DT / NT;        // gate elements per thread
  static_assert((TC * DT) % NT == 0, "the gate pass gives every thread the same number of elements");
  auto gate_elem = [&](int ci, int k, bool live) {
    const unsigned char* stg = smem + (ci % S::NSTAGE) * S::STAGE;
    const T* Xs = reinterpret_cast<const T*>(stg + S::OFF_U);
    const T* DLs = reinterpret_cast<const T*>(stg + S::OFF_DT);
    const T* Zs = reinterpret_cast<const T*>(stg + S::OFF_Z);
    const T* DYs = reinterpret_cast<const T*>(stg + S::OFF_DY);
    const T* YGs = reinterpret_cast<const T*>(stg + S::OFF_YG);
    const int e = tid + k * NT;
    const int t = (ctop - ci) * TC + e / DT, dg = d0 + e % DT;
    const float dyv = to_f32(DYs[e]);
    const float uu = to_f32(Xs[e]);
    // z terms as selects: without z the Z and YG tiles hold stale values that are never
    // selected, and dz is not stored
    const float zz = to_f32(Zs[e]);
    const float sg = sigmoid(zz);
    const float dys = p.has_z ? dyv * zz * sg : dyv;
    st_pred(dz_out + (long long)t * p.dz.sl + dg, from_f32<T>(dyv * to_f32(YGs[e]) * sg * fmaf(zz, 1.0f - sg, 1.0f)),
            live && p.has_z && t < p.L && dg < p.D);   // a warp stores one 32-channel row
    dDacc = live ? fmaf(dys, uu, dDacc) : dDacc;   // thread tid always sees channel tid % 32
    float dtv = to_f32(DLs[e]), sgd = 0.0f;
    if (p.dt_softplus) {                  // rows past L keep delta = 0 (identity steps)
      const float xr = dtv + dtb_gate;
      const bool in = t < p.L;
      dtv = in ? softplus(xr) : 0.0f;
      sgd = in ? sigmoid(xr) : 0.0f;
    }
    SUD[(ci % S::NBUF) * TC * DT + e] = make_float4(uu, dtv, dys, sgd);
  };
  // the state-permuted fp32 copies of chunk ci's B and C: one G-group per thread
  static_assert(2 * TC * N / G == NT, "every thread permutes one G-group of B or C");
  auto permute_bc = [&](int ci) {
    const unsigned char* stg = smem + (ci % S::NSTAGE) * S::STAGE;
    const int e = tid;
    const int which = e / (TC * N / G), r = (e % (TC * N / G)) * G;
    float v[G];
    loadg<G>(reinterpret_cast<const T*>(stg + (which ? S::OFF_C : S::OFF_B)) + r, v);
    float* dst = (which ? SCP : SBP) + (ci % S::NBUF) * G * S::PCP + r;
#pragma unroll
    for (int pm = 0; pm < G; ++pm) {
      float w[G];
#pragma unroll
      for (int j = 0; j < G; ++j) w[j] = v[j ^ pm];
      storeg<G>(dst + pm * S::PCP, w);
    }
  };
  constexpr int GA = S::GA;
  // Prologue: the gate passes of chunks 0 .. GA-1; their stages then take chunks NSTAGE ..
  if constexpr (GA > 0) {
#pragma unroll
    for (int c0 = 0; c0 < GA; ++c0) {
      if (c0 < nch) {
        acquire(c0);
#pragma unroll
        for (int k = 0; k < NE; ++k) gate_elem(c0, k, true);
        permute_bc(c0);
      }
    }
    __syncthreads();
    if (p.use_tma && tid == 0) {
      for (int c0 = S::NSTAGE; c0 < S::NSTAGE + GA && c0 < nch; ++c0)
        bwd_issue_loads<S>(p, smem + (c0 % S::NSTAGE) * S::STAGE, &bars[c0 % S::NSTAGE], d0, (ctop - c0) * TC, b);
    }
  }

  // this thread's coefficient slot of step j: G consecutive floats, 16-byte (G = 4) or 8-byte
  // (G = 2) aligned; a warp's slots of one step are contiguous
  float* const cf_slot = SCF + tid * G;
  constexpr int CF_STEP = NT * G;

  // (3) one recompute step: hc advances by step r of the chunk whose gate products are at
  // (sud, bp); rq / rB hold step r's inputs (fetched one step ahead) and are refilled with step
  // r + 1's.  The step's coefficient goes to the thread's slot for the reverse pass.
  auto rec_step = [&](float2 (&hc)[NP], float4& rq, float2 (&rB)[NP], const float4* sud, const float* bp, int r) {
    const float4 q4 = rq;
    float2 Bn[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) Bn[k] = rB[k];
    if (r + 1 < TC) {
      rq = sud[(r + 1) * DT + dl];
      loadp<G>(bp + (r + 1) * N, rB);
    }
    const float uu = q4.x, dtv = q4.y;
    const float2 u2 = bc2(uu), dt2 = bc2(dtv), dtu2 = bc2(dtv * uu);
    float2 cf[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) {
      if (METHOD == kZOH) {
        const float2 x = mul2(dt2, A2[k]);
        const float2 a = ex2x2(x);
        cf[k] = zoh_r(x, a);                                    // r = A rho = expm1(delta A) - delta A
        hc[k] = fma2(a, hc[k], mul2(fma2(cf[k], iA[k], dt2), mul2(Bn[k], u2)));   // coef = delta + r / A
      } else if (METHOD == kEuler) {
        cf[k] = ex2x2(mul2(dt2, A2[k]));                        // a
        hc[k] = fma2(cf[k], hc[k], mul2(dtu2, Bn[k]));
      } else {
        const float2 zz = mul2(dt2, Ak[k]);
        cf[k] = rcpx2(fma2(bc2(-0.5f), zz, bc2(1.0f)));         // w = 1 / (1 - z/2)
        hc[k] = fma2(mul2(fma2(bc2(0.5f), zz, bc2(1.0f)), cf[k]), hc[k], mul2(mul2(dtu2, Bn[k]), cf[k]));
      }
    }
    if constexpr (S::CACHE) storep<G>(cf_slot + r * CF_STEP, cf);
  };
  auto sud_buf = [&](int ci) { return SUD + (ci % S::NBUF) * TC * DT; };
  auto bp_buf = [&](int ci) { return SBP + (ci % S::NBUF) * G * S::PCP + perm * S::PCP + nbase; };
  // the chunk's states, step by step, from the state entering it
  float2 H[TC][NP];
  auto rec_chunk = [&](const float2 (&h_in)[NP], int ci) {
    float2 hc[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) hc[k] = h_in[k];
    const float4* sud = sud_buf(ci);
    const float* bp = bp_buf(ci);
    float4 rq = sud[dl];                  // step 0's inputs
    float2 rB[NP];
    loadp<G>(bp, rB);
#pragma unroll
    for (int j = 0; j < TC; ++j) {
      rec_step(hc, rq, rB, sud, bp, j);
#pragma unroll
      for (int k = 0; k < NP; ++k) H[j][k] = hc[k];
    }
  };

  auto cs_ptr = [&](int ch) { return p.chunk_states + (((size_t)b * p.nchunks + ch) * p.D + d) * N + nbase; };
  auto cs_load = [&](int ch, float2 (&o)[NP]) {   // the state entering chunk ch (zero before chunk 0)
    if (ch >= 0) {
      slot_load(cs_ptr(ch), o);
    } else {
#pragma unroll
      for (int k = 0; k < NP; ++k) o[k] = bc2(0.f);
    }
  };
  float2 hs[NP];                          // the state entering chunk i
  cs_load(ctop, hs);

  {
    for (int i = 0; i < nch; ++i) {
      const int ch = ctop - i;
      const int t0 = ch * TC;
      float2 hs_next[NP];                 // the state entering chunk i + 1
      cs_load(ch - 1, hs_next);
      if constexpr (GA > 0) {
        if (i + GA < nch) acquire(i + GA);  // consumed by the gate pass inside this chunk's reverse pass
      } else {
        acquire(i);
#pragma unroll
        for (int k = 0; k < NE; ++k) gate_elem(i, k, true);
        permute_bc(i);
        __syncthreads();
      }
      const float4* __restrict__ SUDc = sud_buf(i);
      const float* __restrict__ Bp = bp_buf(i);
      const float* __restrict__ Cp = SCP + (i % S::NBUF) * G * S::PCP + perm * S::PCP + nbase;
      T* const DUo = reinterpret_cast<T*>(smem + S::OFF_OUT + (i % S::NOUT) * 2 * S::OUT);
      T* const DDTo = reinterpret_cast<T*>(smem + S::OFF_OUT + (i % S::NOUT) * 2 * S::OUT + S::OUT);
      rec_chunk(hs, i);

      // (4) reverse adjoint through the chunk.
      float2 pend_b[NP], pend_c[NP];      // the previous step's dB | dC values
      // dB | dC of step js over the warp's channels: slot-splitting stages first (a fixed register
      // slot is sent on every lane thanks to the state permutation), then one stage that splits
      // dB from dC, then all-reduce stages for the remaining channel bits.  Step j's reduction runs
      // after step j - 1's math, so its shuffle latency overlaps work.
      auto reduce_bc = [&](float2 (&xb)[NP], float2 (&xc)[NP], int js) {
        if constexpr (G == 4 && LC >= 1) {   // slot bit 1: keep pair 0, receive the partner's pair 1
          constexpr int m = (CPW / 2) * LPC;
          xb[0] = add2(xb[0], make_float2(__shfl_xor_sync(0xffffffffu, xb[NP - 1].x, m),
                                            __shfl_xor_sync(0xffffffffu, xb[NP - 1].y, m)));
          xc[0] = add2(xc[0], make_float2(__shfl_xor_sync(0xffffffffu, xc[NP - 1].x, m),
                                          __shfl_xor_sync(0xffffffffu, xc[NP - 1].y, m)));
        }
        float keep[BCPL];
        if constexpr (LC >= LG) {            // slot bit 0: (dB, dC) of slot 0
          constexpr int m = (CPW >> LG) * LPC;
          const float2 t2 = add2(make_float2(xb[0].x, xc[0].x),
                                 make_float2(__shfl_xor_sync(0xffffffffu, xb[0].y, m),
                                             __shfl_xor_sync(0xffffffffu, xc[0].y, m)));
          if constexpr (QSTAGE) {
            constexpr int m3 = (CPW >> (LG + 1)) * LPC;
            const bool up = (c >> (LC - LG - 1)) & 1;
            const float send = up ? t2.x : t2.y;
            float kv = (up ? t2.y : t2.x) + __shfl_xor_sync(0xffffffffu, send, m3);
#pragma unroll
            for (int mm = CPW >> (LG + 2); mm >= 1; mm >>= 1) kv += __shfl_xor_sync(0xffffffffu, kv, mm * LPC);
            keep[0] = kv;
          } else {
            keep[0] = t2.x;
            keep[(1) % BCPL] = t2.y;
          }
        } else {                             // CPW = 2, G = 4: slots 0 and 1 remain
          keep[0] = xb[0].x;
          keep[1 % BCPL] = xb[0].y;
          keep[2 % BCPL] = xc[0].x;
          keep[3 % BCPL] = xc[0].y;
        }
        {
          float* dst = SRED + (js * NW + warp) * 2 * N;
          if constexpr (QSTAGE) {
            if ((c & (BCDUP - 1)) == 0) {
              const int q = (c >> (LC - LG - 1)) & 1;
              dst[q * N + nbase + perm] = keep[0];
            }
          } else if constexpr (LC == LG) {
            dst[nbase + perm] = keep[0];
            dst[N + nbase + perm] = keep[1 % BCPL];
          } else {
            dst[nbase + (0 ^ perm)] = keep[0];
            dst[nbase + (1 ^ perm)] = keep[1 % BCPL];
            dst[N + nbase + (0 ^ perm)] = keep[2 % BCPL];
            dst[N + nbase + (1 ^ perm)] = keep[3 % BCPL];
          }
        }
      };
      float4 qn = SUDc[(TC - 1) * DT + dl];   // the last step's inputs, prefetched
      float2 Bnn[NP], Cnn[NP], cfn[NP];
      loadp<G>(Bp + (TC - 1) * N, Bnn);
      loadp<G>(Cp + (TC - 1) * N, Cnn);
      if constexpr (S::CACHE) loadp<G>(cf_slot + (TC - 1) * CF_STEP, cfn);
#pragma unroll
      for (int jg = TC / 4 - 1; jg >= 0; --jg) {
        float red[QV];
#pragma unroll
        for (int jj = 3; jj >= 0; --jj) {
          const int j = jg * 4 + jj;
          // step j's inputs were fetched one step ahead; fetch step j - 1's now
          const float4 q4 = qn;
          float2 Bn[NP], Cn[NP], cf[NP];
#pragma unroll
          for (int k = 0; k < NP; ++k) {
            Bn[k] = Bnn[k];
            Cn[k] = Cnn[k];
            cf[k] = cfn[k];
          }
          if (j > 0) {
            qn = SUDc[(j - 1) * DT + dl];
            loadp<G>(Bp + (j - 1) * N, Bnn);
            loadp<G>(Cp + (j - 1) * N, Cnn);
            if constexpr (S::CACHE) loadp<G>(cf_slot + (j - 1) * CF_STEP, cfn);
          }
          const float uu = q4.x, dtv = q4.y, dys = q4.z;
          const float2 u2 = bc2(uu), dt2 = bc2(dtv), dys2 = bc2(dys);
          if constexpr (!S::CACHE) {        // the recompute pass's coefficients, evaluated again
#pragma unroll
            for (int k = 0; k < NP; ++k) {
              if (METHOD == kZOH) {
                const float2 x = mul2(dt2, A2[k]);
                cf[k] = zoh_r(x, ex2x2(x));
              } else if (METHOD == kEuler) {
                cf[k] = ex2x2(mul2(dt2, A2[k]));
              } else {
                cf[k] = rcpx2(fma2(bc2(-0.5f), mul2(dt2, Ak[k]), bc2(1.0f)));
              }
            }
          }
          float2 duP = bc2(0.f), ddt = bc2(0.f);
          float2 bB[NP], bC[NP];
#pragma unroll
          for (int k = 0; k < NP; ++k) {
            const float2 ht = H[j][k];
            const float2 hp = (j > 0) ? H[j > 0 ? j - 1 : 0][k] : hs[k];
            const float2 Bu = mul2(Bn[k], u2);
            dh[k] = fma2(dys2, Cn[k], dh[k]);
            bC[k] = mul2(dys2, ht);
            if (METHOD == kZOH) {
              // pc = dh coef with coef = expm1(z) / A = delta + r / A, from its two parts
              const float2 dhd = mul2(dh[k], dt2), dhr = mul2(dh[k], cf[k]);
              const float2 pc = fma2(dhr, iA[k], dhd);
              const float2 sv = mul2(dh[k], fma2(Ak[k], ht, Bu));  // dh dh_t/ddelta = dh (A h_t + B u)
              ddt = add2(ddt, sv);
              duP = fma2(pc, Bn[k], duP);
              bB[k] = mul2(pc, u2);
              // A dh dh_t/dA = dh (z h_t - rho B u): dA = sum dh delta h_t - (1/A^2) sum dh r B u
              dAA[k] = fma2(dhd, ht, dAA[k]);
              dAR[k] = fma2(dhr, Bu, dAR[k]);
              dh[k] = fma2(Ak[k], pc, dh[k]);                      // dh a = dh (1 + A coef)
            } else if (METHOD == kEuler) {
              const float2 q = mul2(dh[k], cf[k]);
              const float2 sv = fma2(mul2(q, Ak[k]), hp, mul2(dh[k], Bu));
              ddt = add2(ddt, sv);
              const float2 pc = mul2(dh[k], dt2);
              duP = fma2(pc, Bn[k], duP);
              bB[k] = mul2(pc, u2);
              dAA[k] = fma2(mul2(dt2, q), hp, dAA[k]);
              dh[k] = q;
            } else {
              const float2 w = cf[k];
              const float2 zz = mul2(dt2, Ak[k]);
              const float2 a = mul2(fma2(bc2(0.5f), zz, bc2(1.0f)), w);
              const float2 dhw2 = mul2(mul2(dh[k], w), w);
              const float2 sv = mul2(dhw2, fma2(Ak[k], hp, Bu));
              ddt = add2(ddt, sv);
              const float2 pc = mul2(mul2(dh[k], dt2), w);
              duP = fma2(pc, Bn[k], duP);
              bB[k] = mul2(pc, u2);
              dAA[k] = fma2(mul2(dt2, dhw2), fma2(bc2(0.5f * dtv), Bu, hp), dAA[k]);
              dh[k] = mul2(dh[k], a);
            }
          }
          // step j + 1's dB | dC reduction after step j's math
          if (j < TC - 1) reduce_bc(pend_b, pend_c, j + 1);
#pragma unroll
          for (int k = 0; k < NP; ++k) {
            pend_b[k] = bB[k];
            pend_c[k] = bC[k];
          }
          red[jj * 2 + 0] = duP.x + duP.y;
          red[jj * 2 + 1] = ddt.x + ddt.y;
          if constexpr (GA > 0) {           // a share of chunk i + GA's gate pass (none past the end)
            if (jj == 2) {
              const int q = TC / 4 - 1 - jg;
#pragma unroll
              for (int k = q * NE / 4; k < (q + 1) * NE / 4; ++k) gate_elem(i + GA, k, i + GA < nch);
              if (q == 0) permute_bc(i + GA);
            }
          }
        }
        xpose_reduce<QV, LPC, 1>(red, lane);
        if ((g % QDUP) == 0) {
#pragma unroll
          for (int v = 0; v < QPL; ++v) {
            const int idx = (g / QDUP) * QPL + v;   // value index: step jg*4 + idx/2, quantity idx%2
            const int j = jg * 4 + (idx >> 1);
            if (idx & 1) {
              // chain rule through softplus(raw + bias), as selects (no branch in the unrolled loop)
              const float gs = red[v] * SUDc[j * DT + dl].w;
              DDTo[j * S::OP + dl] = from_f32<T>(p.dt_softplus ? gs : red[v]);
              dtbacc += p.dt_softplus ? gs : 0.0f;
            } else {
              DUo[j * S::OP + dl] = from_f32<T>(fmaf(Dd, SUDc[j * DT + dl].z, red[v]));
            }
          }
        }
      }

      reduce_bc(pend_b, pend_c, 0);       // step 0's dB | dC
      __syncthreads();

      // cross-warp dB | dC sum -> this CTA's partial (fixed order); TC * 2N = G * NT elements
      static_assert(TC * 2 * N == G * NT, "every thread sums G of the chunk's dB | dC values");
#pragma unroll
      for (int k = 0; k < G; ++k) {
        const int e = tid + k * NT;
        const int j = e / (2 * N), v = e % (2 * N);
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) sum += SRED[(j * NW + w) * 2 * N + v];
        const int t = t0 + j;
        st_pred(p.part_bc + (((size_t)b * p.ndt + dtile) * p.L + t) * 2 * N + v, sum, t < p.L);
      }

      if (p.use_tma && tid == 0) {        // the stage just consumed takes chunk nx
        const int nx = i + GA + S::NSTAGE;
        if (nx < nch)
          bwd_issue_loads<S>(p, smem + (nx % S::NSTAGE) * S::STAGE, &bars[nx % S::NSTAGE], d0, (ctop - nx) * TC, b);
      }
      store_tile<NT, S::OP>(DUo, p.du, b, t0, d0, p.L, p.D);
      store_tile<NT, S::OP>(DDTo, p.ddt, b, t0, d0, p.L, p.D);
#pragma unroll
      for (int k = 0; k < NP; ++k) hs[k] = hs_next[k];
    }
  }

  // per-(b, segment, d) partials; ssm_bwd_finalize sums them over (b, segment) in fixed order
  SDD[tid] = dDacc;
  __syncthreads();
  if (dvalid) {
#pragma unroll
    for (int k = 0; k < NP; ++k) {
      const float2 da = (METHOD == kZOH) ? fma2(make_float2(-dAR[k].x, -dAR[k].y), mul2(iA[k], iA[k]), dAA[k]) : dAA[k];
      p.part_A[pbd + ((2 * k) ^ perm)] = da.x;
      p.part_A[pbd + ((2 * k + 1) ^ perm)] = da.y;
      if (p.dh0 != nullptr && seg == 0) {
        p.dh0[bd + ((2 * k) ^ perm)] = dh[k].x;
        p.dh0[bd + ((2 * k + 1) ^ perm)] = dh[k].y;
      }
    }
  }
  if (tid < DT && d0 + tid < p.D) {
    float sdd = 0.f;
    for (int w = 0; w < NT / DT; ++w) sdd += SDD[w * DT + tid];
    p.part_D[bsd * p.D + d0 + tid] = sdd;
  }
  if (p.dt_softplus && p.part_dtb != nullptr) {   // the channel's share sits on its LPC lanes
    const float t = group_allreduce<LPC, 1>(dtbacc);
    if (g == 0 && dvalid) p.part_dtb[bsd * p.D + d] = t;
  }
}

// Sums the per-CTA dB | dC partials over channel tiles and the dA / dD / step-size-bias partials
// over (batch, segment), each in a fixed order (loads of a group of kU terms are issued together, then added in
// index order), and writes dB, dC (element type T), dA, dD, d(bias) (fp32).  dB | dC: one warp per
// (b, t) row, lanes over its 2N values (coalesced, one index division per row); the rest: one
// thread per output.
template <typename T>
__global__ void ssm_bwd_finalize(const FinParams p) {
  constexpr int kU = 8;
  auto sum = [&](const float* src, size_t stride, int cnt) {
    float s = 0.f;
    for (int q0 = 0; q0 < cnt; q0 += kU) {
      float v[kU];
#pragma unroll
      for (int k = 0; k < kU; ++k) v[k] = (q0 + k < cnt) ? __ldg(src + (size_t)(q0 + k) * stride) : 0.f;
#pragma unroll
      for (int k = 0; k < kU; ++k) s += v[k];
    }
    return s;
  };
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const long long gtid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long nthr = (long long)gridDim.x * blockDim.x;
  const int n2 = 2 * p.N;
  const long long rows = (long long)p.B * p.L;
  for (long long r = gtid >> 5; r < rows; r += nthr >> 5) {
    const int b = (int)(r / p.L), t = (int)(r - (long long)b * p.L);
    const float* src = p.part_bc + ((size_t)b * p.ndt * p.L + t) * n2;
    for (int v = lane; v < n2; v += 32) {
      const float s = sum(src + v, (size_t)p.L * n2, p.ndt);
      if (v < p.N) {
        static_cast<T*>(const_cast<void*>(p.dB.ptr))[b * p.dB.sb + (long long)t * p.dB.sl + v] = from_f32<T>(s);
      } else {
        static_cast<T*>(const_cast<void*>(p.dC.ptr))[b * p.dC.sb + (long long)t * p.dC.sl + (v - p.N)] =
            from_f32<T>(s);
      }
    }
  }
  const long long nA = (long long)p.D * p.N;
  const long long nDD = p.dD != nullptr ? p.D : 0;
  const long long total = nA + nDD + (p.ddt_bias != nullptr ? p.D : 0);
  for (long long i = gtid; i < total; i += nthr) {
    if (i < nA) {
      p.dA[i] = sum(p.part_A + i, (size_t)nA, p.nsum);
    } else if (i < nA + nDD) {
      p.dD[i - nA] = sum(p.part_D + (i - nA), (size_t)p.D, p.nsum);
    } else {
      p.ddt_bias[i - nA - nDD] = sum(p.part_dtb + (i - nA - nDD), (size_t)p.D, p.nsum);
    }
  }
}

template <typename T>
cudaError_t launch_bwd(int N, int G, int method, const BwdParams& p, dim3 grid, cudaStream_t stream);
template <typename T>
cudaError_t launch_bwd_finalize(const FinParams& p, cudaStream_t stream);

}  // namespace ssm
