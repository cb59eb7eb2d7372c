// ssm_misc.cu — the single-token state update (decode) and the segment-carry kernel.
#include "ssm_common.cuh"

namespace ssm {

// Composition of per-segment summaries, per (b, d, n):
//   seg_init[s] = carry;  carry = decay[s] * carry + hend[s]       (s = 0 .. S-1)
// or, for the adjoint summaries (reverse), over s = S-1 .. 0.
// The chunk-level combine of the reference's two-level scan (models/scan.py:160-164).  A block owns
// 32 consecutive (b, d, n) columns (coalesced) and kCarryGroups groups of consecutive segments
// (threadIdx.y): every group composes its segments into one (decay, end) pair, the groups' pairs are
// composed in order by one thread per column, and every group then walks its segments again from
// its carried-in value.  Two passes over the summaries, but kCarryGroups times the loads in flight
// of a one-thread-per-column walk, which is latency-bound (148 segments: ~30 us).
constexpr int kCarryGroups = 16;
__global__ void __launch_bounds__(32 * kCarryGroups) ssm_carry_kernel(const CarryParams p) {
  __shared__ float s_dec[kCarryGroups][32], s_end[kCarryGroups][32], s_in[kCarryGroups][32];
  pdl_launch_dependents();
  pdl_wait();
  const long long dn_total = (long long)p.D * p.N;
  const long long idx = blockIdx.x * 32LL + threadIdx.x;
  const bool live = idx < (long long)p.B * dn_total;
  const long long b = live ? idx / dn_total : 0, dn = live ? idx % dn_total : 0;
  const size_t base = (size_t)b * p.nseg * dn_total + dn;
  const int grp = threadIdx.y;
  const int per = (p.nseg + kCarryGroups - 1) / kCarryGroups;
  const int i0 = grp * per, i1 = min(p.nseg, i0 + per);          // processing positions [i0, i1)
  auto seg_at = [&](int i) { return p.reverse ? p.nseg - 1 - i : i; };
  float dec = 1.0f, end = 0.0f;
  if (live) {
#pragma unroll 4
    for (int i = i0; i < i1; ++i) {
      const size_t o = base + (size_t)seg_at(i) * dn_total;
      const float a = p.seg_decay[o];
      end = fmaf(a, end, p.seg_hend[o]);
      dec *= a;
    }
  }
  s_dec[grp][threadIdx.x] = dec;
  s_end[grp][threadIdx.x] = end;
  __syncthreads();
  if (grp == 0) {
    float carry = (live && p.h_init != nullptr) ? p.h_init[idx] : 0.0f;
    float tot = 1.0f;
    for (int g2 = 0; g2 < kCarryGroups; ++g2) {
      s_in[g2][threadIdx.x] = carry;
      carry = fmaf(s_dec[g2][threadIdx.x], carry, s_end[g2][threadIdx.x]);
      tot *= s_dec[g2][threadIdx.x];
    }
    if (live && p.tot_hend != nullptr) p.tot_hend[idx] = carry;
    if (live && p.tot_decay != nullptr) p.tot_decay[idx] = tot;
  }
  __syncthreads();
  if (live && p.seg_init != nullptr) {
    float carry = s_in[grp][threadIdx.x];
#pragma unroll 4
    for (int i = i0; i < i1; ++i) {
      const size_t o = base + (size_t)seg_at(i) * dn_total;
      p.seg_init[o] = carry;
      carry = fmaf(p.seg_decay[o], carry, p.seg_hend[o]);
    }
  }
}

cudaError_t launch_carry(const CarryParams& p, cudaStream_t stream) {
  const long long total = (long long)p.B * p.D * p.N;
  return launch_pdl(ssm_carry_kernel, dim3((unsigned)((total + 31) / 32)), dim3(32, kCarryGroups), 0, stream, p);
}

// Composition of W shard summaries (shard r's (B, D, N) block at r * stride elements), one thread
// per (b, d, n):
//   out[r] = carry;  carry = decay[r] * carry + end[r]        (r = 0 .. W-1, or W-1 .. 0 reversed)
// with carry starting at start (or 0); the final carry goes to last.  The cross-GPU form of the
// segment carry above: the prefix of the sequence-sharded forward (the carried-in state of every
// shard) and the suffix of its backward (the adjoint entering every shard), one launch instead of
// two small tensor operations per shard.
__global__ void ssm_compose_kernel(const float* __restrict__ decay, const float* __restrict__ end,
                                   const float* __restrict__ start, float* __restrict__ out,
                                   float* __restrict__ last, int W, long long elems, long long stride, int reverse) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= elems) return;
  float carry = start != nullptr ? start[i] : 0.0f;
  for (int k = 0; k < W; ++k) {
    const long long r = reverse ? W - 1 - k : k;
    const long long o = r * stride + i;
    out[r * elems + i] = carry;
    carry = fmaf(decay[o], carry, end[o]);
  }
  if (last != nullptr) last[i] = carry;
}

cudaError_t launch_compose(const float* decay, const float* end, const float* start, float* out, float* last, int W,
                           long long elems, long long stride, int reverse, cudaStream_t stream) {
  const unsigned blocks = (unsigned)((elems + 255) / 256);
  ssm_compose_kernel<<<blocks, 256, 0, stream>>>(decay, end, start, out, last, W, elems, stride, reverse);
  return cudaGetLastError();
}

// Single-token state update: the inline decode branch of Mamba.forward
// (models/mamba.py:113-118, 123-124).  LPC = N/4 lanes per channel, 4 states per lane.
template <int N, typename T>
__global__ void __launch_bounds__(128) ssm_update_kernel(const UpdParams p) {
  constexpr int LPC = N / 4;
  const long long gt = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long chn = gt / LPC;
  const int g = (int)(gt % LPC);
  const bool valid = chn < (long long)p.B * p.D;
  const int b = valid ? (int)(chn / p.D) : 0;
  const int d = valid ? (int)(chn % p.D) : 0;
  float h[4] = {0.f, 0.f, 0.f, 0.f}, Ak[4] = {-1.f, -1.f, -1.f, -1.f}, Bn[4] = {0.f, 0.f, 0.f, 0.f},
        Cn[4] = {0.f, 0.f, 0.f, 0.f};
  float xv = 0.f, dtv = 0.f;
  float* hp = p.state + ((size_t)b * p.D + d) * N + g * 4;
  if (valid) {
    load4(hp, h);
    load4(p.A + (size_t)d * N + g * 4, Ak);
    const T* Bm = static_cast<const T*>(p.Bm.ptr) + b * p.Bm.sb + g * 4;
    const T* Cm = static_cast<const T*>(p.Cm.ptr) + b * p.Cm.sb + g * 4;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      Bn[k] = to_f32(Bm[k]);
      Cn[k] = to_f32(Cm[k]);
    }
    xv = to_f32(static_cast<const T*>(p.x.ptr)[b * p.x.sb + d]);
    dtv = to_f32(static_cast<const T*>(p.dt.ptr)[b * p.dt.sb + d]);
  }
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float z = dtv * Ak[k];
    float a, bb;
    if (p.method == kZOH) {
      const float x = z * kLog2e;
      a = ex2(x);
      bb = em1x(x, a) / Ak[k] * (Bn[k] * xv);   // expm1(delta A) / A B x, accurate for small |delta A|
    } else if (p.method == kEuler) {
      a = ex2(z * kLog2e);
      bb = dtv * (Bn[k] * xv);
    } else {
      const float w = 1.0f / (1.0f - 0.5f * z);
      a = (1.0f + 0.5f * z) * w;
      bb = dtv * w * (Bn[k] * xv);
    }
    h[k] = fmaf(a, h[k], bb);
    acc = fmaf(Cn[k], h[k], acc);
  }
#pragma unroll
  for (int m = LPC / 2; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
  if (valid) {
    *reinterpret_cast<float4*>(hp) = make_float4(h[0], h[1], h[2], h[3]);
    if (g == 0) {
      float yv = acc;
      if (p.Dskip != nullptr) yv = fmaf(p.Dskip[d], xv, yv);
      if (p.has_z) {
        const float zz = to_f32(static_cast<const T*>(p.z.ptr)[b * p.z.sb + d]);
        yv *= zz * sigmoid(zz);
      }
      static_cast<T*>(const_cast<void*>(p.y.ptr))[b * p.y.sb + d] = from_f32<T>(yv);
    }
  }
}

template <typename T>
static cudaError_t launch_update_t(int N, const UpdParams& p, cudaStream_t stream) {
  const long long threads = (long long)p.B * p.D * (N / 4);
  const unsigned blocks = (unsigned)((threads + 127) / 128);
  switch (N) {
    case 4: ssm_update_kernel<4, T><<<blocks, 128, 0, stream>>>(p); break;
    case 8: ssm_update_kernel<8, T><<<blocks, 128, 0, stream>>>(p); break;
    case 16: ssm_update_kernel<16, T><<<blocks, 128, 0, stream>>>(p); break;
    case 32: ssm_update_kernel<32, T><<<blocks, 128, 0, stream>>>(p); break;
    case 64: ssm_update_kernel<64, T><<<blocks, 128, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_update(int N, bool bf16, const UpdParams& p, cudaStream_t stream) {
  return bf16 ? launch_update_t<__nv_bfloat16>(N, p, stream) : launch_update_t<float>(N, p, stream);
}

}  // namespace ssm
