// ssm_common.cuh — device helpers and launch geometry shared by the selective-scan kernels.
//
// Geometry (all scan kernels): one thread owns G consecutive states (n = G g .. G g + G-1) of
// one channel (G = 4, or G = 2 when the (batch x channel) grid is too small to fill the GPU);
// N/G consecutive lanes ("a channel group") cover all N states of a channel, so a warp covers
// 32 G / N channels and a CTA of N/G warps covers DT = 32 channels.  Time is walked
// sequentially in tiles of TC = 16 steps that TMA stages into shared memory.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace ssm {

constexpr float kLog2e = 1.4426950408889634f;

enum { kZOH = 0, kEuler = 1, kBilinear = 2 };

template <int N_, int G_ = 4>
struct Geo {
  static constexpr int N = N_;
  static constexpr int G = G_;             // states per thread
  static constexpr int LPC = N / G;        // lanes per channel
  static constexpr int CPW = 32 / LPC;     // channels per warp
  static constexpr int DT = 32;            // channels per CTA
  static constexpr int NW = DT / CPW;      // warps per CTA (= N / G)
  static constexpr int NT = NW * 32;       // threads per CTA (= 32 N / G)
  static constexpr int TC = 16;            // time steps per tile (= checkpoint interval)
  static_assert((G == 2 || G == 4) && N % G == 0 && LPC >= 1 && LPC <= 16, "unsupported N / G");
};

constexpr int kChunk = 16;  // checkpoint interval of chunk_states (time steps)

// ------------------------------------------------------------------------------------------
// Element access
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float x) { return x; }
// 4 consecutive elements (16-byte aligned for float, 8-byte aligned for bf16) as float.
__device__ __forceinline__ void load4(const float* p, float (&o)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&o)[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  o[0] = __uint_as_float(v.x << 16); o[1] = __uint_as_float(v.x & 0xffff0000u);
  o[2] = __uint_as_float(v.y << 16); o[3] = __uint_as_float(v.y & 0xffff0000u);
}
__device__ __forceinline__ void load2(const float* p, float (&o)[2]) {
  const float2 v = *reinterpret_cast<const float2*>(p);
  o[0] = v.x; o[1] = v.y;
}
__device__ __forceinline__ void load2(const __nv_bfloat16* p, float (&o)[2]) {
  const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
  o[0] = __uint_as_float(v << 16); o[1] = __uint_as_float(v & 0xffff0000u);
}
// G consecutive values (G = 2 or 4) as float; p aligned to G elements.
template <int G, typename T>
__device__ __forceinline__ void loadg(const T* p, float (&o)[G]) {
  if constexpr (G == 4) load4(p, o);
  else load2(p, o);
}
template <int G>
__device__ __forceinline__ void storeg(float* p, const float (&v)[G]) {
  if constexpr (G == 4) *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  else *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
}
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Global store under a predicate, as one predicated instruction (no branch, so the unrolled loop it
// sits in stays one basic block for the scheduler).
__device__ __forceinline__ void st_pred(float* ptr, float v, bool ok) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %2, 0;\n\t@p st.global.f32 [%0], %1;\n\t}" ::"l"(ptr), "f"(v),
               "r"((int)ok));
}
__device__ __forceinline__ void st_pred(__nv_bfloat16* ptr, __nv_bfloat16 v, bool ok) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %2, 0;\n\t@p st.global.b16 [%0], %1;\n\t}" ::"l"(ptr),
               "h"(__bfloat16_as_ushort(v)), "r"((int)ok));
}
// 2^x on the MUFU unit (flush-to-zero for subnormal results: the decays are in (0, 1]).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Packed pair arithmetic (FFMA2 / FMUL2 / FADD2 on sm_100): one instruction for two states.
__device__ __forceinline__ float2 bc2(float x) { return make_float2(x, x); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 ex2x2(float2 x) { return make_float2(ex2(x.x), ex2(x.y)); }
__device__ __forceinline__ float2 rcpx2(float2 x) { return make_float2(rcp(x.x), rcp(x.y)); }
// G consecutive values as G/2 pairs
template <int G, typename T>
__device__ __forceinline__ void loadp(const T* p, float2 (&o)[G / 2]) {
  float v[G];
  loadg<G>(p, v);
#pragma unroll
  for (int i = 0; i < G / 2; ++i) o[i] = make_float2(v[2 * i], v[2 * i + 1]);
}
template <int G>
__device__ __forceinline__ void storep(float* p, const float2 (&v)[G / 2]) {
  if constexpr (G == 4) *reinterpret_cast<float4*>(p) = make_float4(v[0].x, v[0].y, v[1].x, v[1].y);
  else *reinterpret_cast<float2*>(p) = v[0];
}

// 2^x - 1 for a pair, given a = ex2(x) from the MUFU: the ZOH input coefficient
// expm1(delta A) (models/scan.py:50 uses torch.expm1), accurate in relative terms also where |x|
// is small.  a - 1 alone is not: ex2.approx's absolute error near 1 (about 1e-7) becomes a
// relative error of about 1e-7 / |delta A| in expm1, 1e-3 at |delta A| = 1e-4.
// Both candidates are lower bounds of e^z - 1 (z = x ln 2) for every x:
//   * the third-order Taylor polynomial z + z^2/2 + z^3/6 (Lagrange remainder e^xi z^4/24 >= 0);
//   * the MUFU value scaled down by (1 - 2^-22), more than ex2.approx's relative error (measured
//     on B200 against double-precision exp2: at most 1.46e-7 = 2^-22.7 over every float in
//     [-1, 1] and a sample of [-126, 64)), minus 1.
// Their maximum is therefore within min(z^4/24, 3.9e-7 e^z) of e^z - 1: the polynomial wins for
// small |z|, the MUFU value for large |z|, and the worst relative error (|z| near 0.055) is about
// 7e-6.  Five FP operations per pair beyond a - 1; no branch, no division.
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kEm1C1 = kLn2;                                 // ln2
constexpr float kEm1C2 = 0.2402265069591007f;                  // ln2^2 / 2
constexpr float kEm1C3 = 0.05550410866482158f;                 // ln2^3 / 6
constexpr float kEm1Scale = 1.0f - 2.384185791015625e-7f;      // 1 - 2^-22
__device__ __forceinline__ float2 em1x2(float2 x, float2 a) {
  const float2 e = fma2(a, bc2(kEm1Scale), bc2(-1.0f));
  float2 p = fma2(x, bc2(kEm1C3), bc2(kEm1C2));
  p = fma2(x, p, bc2(kEm1C1));
  const float2 s = mul2(x, p);
  return make_float2(fmaxf(s.x, e.x), fmaxf(s.y, e.y));
}
__device__ __forceinline__ float em1x(float x, float a) {
  const float e = fmaf(a, kEm1Scale, -1.0f);
  const float s = x * fmaf(x, fmaf(x, kEm1C3, kEm1C2), kEm1C1);
  return fmaxf(s, e);
}

// logistic sigmoid from e^-z = 2^(-z log2 e)
__device__ __forceinline__ float sigmoid(float z) { return rcp(1.0f + ex2(-z * kLog2e)); }
// softplus(x) = log(1 + e^x) with torch's default threshold (x > 20 returns x), the step-size
// activation of models/mamba.py:77: max(x, 0) + log1p(e^-|x|)
__device__ __forceinline__ float softplus(float x) {
  return x > 20.0f ? x : fmaxf(x, 0.0f) + log1pf(__expf(-fabsf(x)));
}

// ------------------------------------------------------------------------------------------
// Warp transposition-reduce.  v[0..V) hold this lane's partial sums of V quantities; the
// GROUP lanes {l, l ^ STRIDE, l ^ 2 STRIDE, ...} each contribute one partial per quantity.
// Recursive halving: at every stage a lane keeps half of its live values and sends the other
// half to its partner, so V values are reduced over GROUP lanes with (V - V/GROUP) shuffles
// instead of V log2(GROUP).  On return, with r = (lane / STRIDE) % GROUP:
//   V >= GROUP: v[0 .. V/GROUP) hold quantities [r V/GROUP, (r+1) V/GROUP)
//   V <  GROUP: v[0] holds quantity r / (GROUP / V)  (duplicated on GROUP/V lanes)
// V and GROUP are powers of two.
// ------------------------------------------------------------------------------------------
template <int V, int GROUP, int STRIDE>
__device__ __forceinline__ void xpose_reduce(float (&v)[V], int lane) {
  static_assert((V & (V - 1)) == 0 && (GROUP & (GROUP - 1)) == 0, "powers of two");
#pragma unroll
  for (int stage = 0; (GROUP >> (stage + 1)) >= 1; ++stage) {
    const int m = (GROUP >> (stage + 1)) * STRIDE;
    const int K = V >> stage;
    if (K >= 2) {
      const int half = K >> 1;
      const bool upper = (lane & m) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = upper ? v[i] : v[i + half];
        const float keep = upper ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
    }
  }
}

// Plain butterfly all-reduce of one value over GROUP lanes spaced STRIDE apart.
template <int GROUP, int STRIDE>
__device__ __forceinline__ float group_allreduce(float x) {
#pragma unroll
  for (int m = GROUP / 2; m >= 1; m >>= 1) x += __shfl_xor_sync(0xffffffffu, x, m * STRIDE);
  return x;
}

struct DAct {                // (B, rows, cols) tensor with unit column stride
  const void* ptr;
  long long sb, sl;          // element strides of batch and row
};

// Row pitch (in elements of T) of a padded (16 x 32) shared tile written or read in blocks of
// LPC rows x CPW consecutive channels: consecutive rows start SW 4-byte words apart, SW >= the
// block's width in words and a multiple of 4, so rows stay 16-byte aligned (vector copies) and
// a block spreads over the 32 banks (2-way overlap remains only for CPW = 2).
template <int CPW, typename T>
struct PadPitch {
  static constexpr int WW = CPW * (int)sizeof(T) / 4 > 0 ? CPW * (int)sizeof(T) / 4 : 1;
  static constexpr int SW = WW < 4 ? 4 : WW;
  static constexpr int value = 32 + SW * 4 / (int)sizeof(T);
  static_assert((value * (int)sizeof(T)) % 16 == 0, "padded rows must stay 16-byte aligned");
};

// Coalesced copy of a padded (16 x OP) shared tile to a (B, L, D) view (16-byte stores
// where the row and view allow it).
template <int NT, int OP, typename T>
__device__ __forceinline__ void store_tile(const T* tile, const DAct& v, int b, int t0, int d0, int L, int D) {
  constexpr int TC = 16, DT = 32, VEC = 16 / (int)sizeof(T);   // elements per 16 bytes
  static_assert((OP * (int)sizeof(T)) % 16 == 0, "16-byte shared loads need 16-byte aligned rows");
  T* base = static_cast<T*>(const_cast<void*>(v.ptr)) + b * v.sb;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(base) | (uintptr_t)(v.sl * sizeof(T))) & 15) == 0 &&
                      (d0 + DT <= D);
  if (vec_ok) {
    for (int e = threadIdx.x; e < TC * DT / VEC; e += NT) {
      const int tt = e / (DT / VEC), q = e % (DT / VEC);
      if (t0 + tt < L)
        *reinterpret_cast<uint4*>(base + (long long)(t0 + tt) * v.sl + d0 + q * VEC) =
            *reinterpret_cast<const uint4*>(tile + tt * OP + q * VEC);
    }
  } else {
    for (int e = threadIdx.x; e < TC * DT; e += NT) {
      const int tt = e / DT, dd = e % DT;
      if (t0 + tt < L && d0 + dd < D) base[(long long)(t0 + tt) * v.sl + d0 + dd] = tile[tt * OP + dd];
    }
  }
}

// ------------------------------------------------------------------------------------------
// mbarrier + TMA (cp.async.bulk.tensor) wrappers.  No cluster multicast anywhere.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// Programmatic dependent launch.  A kernel launched with launch_pdl may be scheduled while the
// kernel before it in the stream is still draining.  Every such kernel calls pdl_wait() before its
// first global-memory access (read or write): it returns once the previous kernel has completed
// and its writes are visible, so the kernel sees exactly what a plain launch would see.
// pdl_launch_dependents() at a kernel's top lets the next launch_pdl kernel be scheduled once all
// of this grid's CTAs are running.  Kernels from other libraries that follow are launched
// normally.  Measured at config 1 (fwd + bwd + finalize): 173.3 -> 171.3 us per step.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after ~2^24 polls (seconds), records the failure in *err and
// returns, so a copy that never lands ends the kernel with an error flag instead of a hang.
__device__ __forceinline__ void mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t it = 0; it < (1u << 24); ++it) {
    if (mbar_try_wait(bar, parity)) return;
  }
  if (err) atomicOr(err, 1);
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 3-D tiled TMA load into shared memory, completion signalled on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}
// 3-D tiled TMA store from shared memory (out-of-range parts of the box are not written).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int Pending>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(Pending) : "memory");
}
template <int Pending>
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(Pending) : "memory");
}

// ------------------------------------------------------------------------------------------
// Kernel parameter blocks (passed as __grid_constant__ so the tensor maps stay addressable)
// ------------------------------------------------------------------------------------------

struct alignas(64) FwdParams {
  CUtensorMap tm_u, tm_dt, tm_z, tm_B, tm_C;        // TMA loads (outputs use plain stores)
  DAct u, dt, z, Bm, Cm, y, yg;   // yg: pre-gate output (y + Dskip u), written iff save_ygate
  const float* A;            // (D, N)
  const float* Dskip;        // (D) or null
  const float* h_init;       // (B, D, N) or null: state entering t = 0 (segment 0)
  const float* seg_init;     // (B, S, D, N) or null: state entering each segment (S > 1)
  float* last;               // (B, D, N) or null
  float* chunk_states;       // (B, nchunks, D, N) or null
  float* seg_hend;           // summary mode: (B, S, D, N)
  float* seg_decay;          // summary mode: (B, S, D, N)
  const float* dt_bias;      // (D) or null: added to delta before the softplus
  int* err;
  int B, L, D, nchunks, seg_len, nseg;
  int seg_first;             // segment of blockIdx.y = 0 (grids over a suffix of the segments)
  int has_z, use_tma, save_ygate;
  int dt_softplus;           // delta = softplus(delta + dt_bias) in the kernel
};

struct alignas(64) BwdParams {
  CUtensorMap tm_u, tm_dt, tm_z, tm_dy, tm_yg, tm_B, tm_C;   // TMA loads (outputs use plain stores)
  DAct u, dt, z, dy, yg, Bm, Cm, du, ddt, dz;   // yg: the forward's pre-gate output (iff has_z)
  const float* A;
  const float* Dskip;
  const float* h0;           // (B, D, N) or null (only for dh0 presence)
  const float* chunk_states; // (B, nchunks, D, N)
  const float* dlast;        // (B, D, N) or null
  const float* seg_dh;       // (B, S, D, N) or null: the adjoint entering each segment from its right (S > 1)
  float* dh0;                // (B, D, N) or null
  float* part_bc;            // (B, nDT, L, 2N): per-CTA dB | dC partial sums
  float* part_A;             // (B, S, D, N)
  float* part_D;             // (B, S, D)
  const float* dt_bias;      // (D) or null (see FwdParams)
  float* part_dtb;           // (B, S, D): per-(batch, segment) sums of the raw-delta gradient (dt_softplus)
  int* err;
  int B, L, D, nchunks, ndt;
  int nseg, seg_len;         // sequence segments (blockIdx.z) of seg_len steps, a multiple of 16
  int has_z, use_tma;
  int dt_softplus;           // ddt is then the gradient w.r.t. the raw delta: ddelta * sigmoid(raw + bias)
};

struct FinParams {
  const float* part_bc;
  const float* part_A;
  const float* part_D;
  DAct dB, dC;               // outputs (B, L, N), element type T
  float* dA;                 // (D, N)
  float* dD;                 // (D) or null
  const float* part_dtb;     // (B, S, D) or null
  float* ddt_bias;           // (D) or null
  int B, L, D, N, ndt;
  int nsum;                  // partial groups of dA, dD, d(bias): B x backward segments
};

struct CarryParams {
  const float* h_init;       // (B, D, N) or null
  const float* seg_decay;    // (B, S, D, N)
  const float* seg_hend;     // (B, S, D, N)
  float* seg_init;           // (B, S, D, N) or null
  float* tot_decay;          // (B, D, N) or null
  float* tot_hend;           // (B, D, N) or null
  int B, D, N, nseg;
  int reverse;               // compose from the last segment to the first (adjoint summaries)
};

struct UpdParams {
  float* state;              // (B, D, N)
  DAct x, dt, Bm, Cm, z, y;  // sb used, sl ignored
  const float* A;
  const float* Dskip;
  int B, D, method, has_z;
};

}  // namespace ssm
