// ssm_conv.cu — causal depthwise conv1d + SiLU, forward and backward: the step in front of the
// selective scan in the Mamba mixer.
//
// Replaces models/mamba.py:100-107: x (B, L, D) is transposed to (B, D, L), left-padded with
// d_conv - 1 zeros (or prefixed with the decode state's last d_conv - 1 inputs), passed through
// nn.Conv1d(D, D, K, groups=D) and SiLU, and transposed back.  Here the (B, L, D) layout is read
// and written directly (x may be a strided view, e.g. the first half of in_proj's output), with
//   out[b, t, d] = silu(bias[d] + sum_k w[d, k] x[b, t - (K - 1) + k, d]),   x[t < 0] = state.
// Every thread owns VEC consecutive channels of one time tile and slides a K - 1 row window down
// the tile, so each input row is read once per tile (plus a K - 1 row halo) with 16-byte loads.
//
// Backward: g = dout silu'(pre) is recomputed row by row; dx[s] = sum_k w[k] g[s + K - 1 - k]
// (a K - 1 row look-ahead past the tile), and the weight / bias gradients are summed per thread
// over its tile and then over (batch, tile) in a fixed order by a second kernel: deterministic,
// no float atomics.
#include <cuda_runtime.h>

#include <cstdio>

#include "ssm_b200.h"
#include "ssm_common.cuh"

namespace ssm {
int report_error(int code, const char* msg);
}  // namespace ssm

namespace {

using ssm::from_f32;
using ssm::to_f32;

constexpr int kThreads = 128;
constexpr int kU = 4;          // rows loaded per round by each thread
constexpr int kTTMax = 64;     // time steps per tile, at most (tiles are shortened for small grids)

struct ConvParams {
  const void* x;
  long long xsb, xsl;
  void* out;                   // forward: out; backward: dx
  long long osb, osl;
  const void* dout;            // backward only
  long long gsb, gsl;
  const float* w;              // (D, K)
  const float* bias;           // (D) or null
  const void* state;           // (B, D, K - 1) in x's dtype, or null
  void* new_state;             // (B, D, K - 1) or null
  float* part;                 // backward: (B, ntile, D, K + 1) partial sums
  float* dw;
  float* db;
  int B, L, D, ntile, tt, silu;
};

// Tile length: the longest power of two <= 64 that still gives about 4 CTAs per SM (each tile
// costs a K - 1 row halo, so long tiles are cheaper when the grid is large enough).
int tile_len(int64_t B, int64_t L, int64_t D, int vec) {
  const int64_t ctas_per_tile_row = B * ((D / vec + kThreads - 1) / kThreads);
  int tt = kTTMax;
  while (tt > 4 && ctas_per_tile_row * ((L + tt - 1) / tt) < 4 * 148) tt /= 2;
  return tt;
}

template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const T* src, float (&v)[VEC]) {
  if constexpr (VEC == 1) {
    v[0] = to_f32(src[0]);
  } else if constexpr (sizeof(T) == 4) {
    static_assert(VEC == 4, "fp32 vectors are 4 wide");
    const float4 q = *reinterpret_cast<const float4*>(src);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  } else {
    static_assert(VEC == 8, "bf16 vectors are 8 wide");
    const uint4 q = *reinterpret_cast<const uint4*>(src);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T* dst, const float (&v)[VEC]) {
  if constexpr (VEC == 1) {
    dst[0] = from_f32<T>(v[0]);
  } else if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    uint4 q;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(dst) = q;
  }
}

template <typename T, int VEC, int K>
__global__ void __launch_bounds__(kThreads) conv_fwd_kernel(const ConvParams p) {
  const int d0 = (blockIdx.x * kThreads + threadIdx.x) * VEC;
  if (d0 >= p.D) return;
  const int b = blockIdx.z, t0 = blockIdx.y * p.tt, t1 = min(p.L, t0 + p.tt);
  const T* xb = static_cast<const T*>(p.x) + b * p.xsb + d0;
  T* ob = static_cast<T*>(p.out) + b * p.osb + d0;
  float w[K][VEC], bias[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
#pragma unroll
    for (int k = 0; k < K; ++k) w[k][v] = p.w[(size_t)(d0 + v) * K + k];
    bias[v] = p.bias != nullptr ? p.bias[d0 + v] : 0.0f;
  }
  // window: inputs at t0 - (K - 1) .. t0 - 1 (the decode state, or zeros, before t = 0)
  float win[K > 1 ? K - 1 : 1][VEC];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const int t = t0 - (K - 1) + j;
    if (t >= 0) {
      load_vec<T, VEC>(xb + (long long)t * p.xsl, win[j]);
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v)
        win[j][v] = p.state != nullptr
                        ? to_f32(static_cast<const T*>(p.state)[((size_t)b * p.D + d0 + v) * (K - 1) + (K - 1 + t)])
                        : 0.0f;
    }
  }
  // kU rows per round: their loads are issued together, so each thread keeps kU rows in flight
  for (int tr = t0; tr < t1; tr += kU) {
    float xr[kU][VEC];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (tr + u < t1) load_vec<T, VEC>(xb + (long long)(tr + u) * p.xsl, xr[u]);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (tr + u >= t1) break;
      float o[VEC];
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        float acc = fmaf(w[K - 1][v], xr[u][v], bias[v]);
#pragma unroll
        for (int j = 0; j < K - 1; ++j) acc = fmaf(w[j][v], win[j][v], acc);
        o[v] = p.silu ? acc * ssm::sigmoid(acc) : acc;
      }
      store_vec<T, VEC>(ob + (long long)(tr + u) * p.osl, o);
#pragma unroll
      for (int j = 0; j + 1 < K - 1; ++j)
#pragma unroll
        for (int v = 0; v < VEC; ++v) win[j][v] = win[j + 1][v];
      if (K > 1) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) win[K > 1 ? K - 2 : 0][v] = xr[u][v];
      }
    }
  }
  // the last tile leaves the last K - 1 inputs of cat(state, x) as the new decode state
  if (p.new_state != nullptr && t1 == p.L) {
#pragma unroll
    for (int j = 0; j < K - 1; ++j)
#pragma unroll
      for (int v = 0; v < VEC; ++v)
        static_cast<T*>(p.new_state)[((size_t)b * p.D + d0 + v) * (K - 1) + j] = from_f32<T>(win[j][v]);
  }
}

template <typename T, int VEC, int K>
__global__ void __launch_bounds__(kThreads) conv_bwd_kernel(const ConvParams p) {
  const int d0 = (blockIdx.x * kThreads + threadIdx.x) * VEC;
  if (d0 >= p.D) return;
  const int b = blockIdx.z, tile = blockIdx.y, t0 = tile * p.tt, t1 = min(p.L, t0 + p.tt);
  const T* xb = static_cast<const T*>(p.x) + b * p.xsb + d0;
  const T* gb = static_cast<const T*>(p.dout) + b * p.gsb + d0;
  T* dxb = static_cast<T*>(p.out) + b * p.osb + d0;
  float w[K][VEC], bias[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
#pragma unroll
    for (int k = 0; k < K; ++k) w[k][v] = p.w[(size_t)(d0 + v) * K + k];
    bias[v] = p.bias != nullptr ? p.bias[d0 + v] : 0.0f;
  }
  float xw[K > 1 ? K - 1 : 1][VEC], gq[K > 1 ? K - 1 : 1][VEC], dw[K][VEC], dbs[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    dbs[v] = 0.0f;
#pragma unroll
    for (int k = 0; k < K; ++k) dw[k][v] = 0.0f;
#pragma unroll
    for (int j = 0; j < K - 1; ++j) gq[j][v] = 0.0f;
  }
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const int t = t0 - (K - 1) + j;
    if (t >= 0) {
      load_vec<T, VEC>(xb + (long long)t * p.xsl, xw[j]);
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) xw[j][v] = 0.0f;
    }
  }
  // rows t0 .. t1 + K - 2: g of every row; dx of row t - (K - 1) once its look-ahead is complete
  const int tend = t1 + K - 1;
  for (int tr = t0; tr < tend; tr += kU) {
    // kU rows per round: their loads are issued together (rows past L read nothing)
    float xr[kU][VEC], dr[kU][VEC];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (tr + u < tend && tr + u < p.L) {
        load_vec<T, VEC>(xb + (long long)(tr + u) * p.xsl, xr[u]);
        load_vec<T, VEC>(gb + (long long)(tr + u) * p.gsl, dr[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tr + u;
      if (t >= tend) break;
      const bool valid = t < p.L;
      float xv[VEC], gv[VEC];
      if (valid) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) xv[v] = xr[u][v];
        const float (&dv)[VEC] = dr[u];
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          float pre = fmaf(w[K - 1][v], xv[v], bias[v]);
#pragma unroll
          for (int j = 0; j < K - 1; ++j) pre = fmaf(w[j][v], xw[j][v], pre);
          if (p.silu) {
            const float s = ssm::sigmoid(pre);
            gv[v] = dv[v] * s * fmaf(pre, 1.0f - s, 1.0f);
          } else {
            gv[v] = dv[v];
          }
        }
      } else {
#pragma unroll
        for (int v = 0; v < VEC; ++v) xv[v] = gv[v] = 0.0f;
      }
      if (t < t1) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          dbs[v] += gv[v];
#pragma unroll
          for (int j = 0; j < K - 1; ++j) dw[j][v] = fmaf(gv[v], xw[j][v], dw[j][v]);
          dw[K - 1][v] = fmaf(gv[v], xv[v], dw[K - 1][v]);
        }
      }
      const int s = t - (K - 1);
      if (s >= t0 && s < t1) {       // dx[s] = sum_k w[k] g[s + K - 1 - k]; g[t] is the newest
        float o[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          float acc = w[0][v] * gv[v];
#pragma unroll
          for (int k = 1; k < K; ++k) acc = fmaf(w[k][v], gq[K - 1 - k][v], acc);
          o[v] = acc;
        }
        store_vec<T, VEC>(dxb + (long long)s * p.osl, o);
      }
#pragma unroll
      for (int j = 0; j + 1 < K - 1; ++j)
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          xw[j][v] = xw[j + 1][v];
          gq[j][v] = gq[j + 1][v];
        }
      if (K > 1) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          xw[K > 1 ? K - 2 : 0][v] = xv[v];
          gq[K > 1 ? K - 2 : 0][v] = gv[v];
        }
      }
    }
  }
  float* part = p.part + (((size_t)b * p.ntile + tile) * p.D + d0) * (K + 1);
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
#pragma unroll
    for (int k = 0; k < K; ++k) part[v * (K + 1) + k] = dw[k][v];
    part[v * (K + 1) + K] = dbs[v];
  }
}

// dweight (D, K) and dbias (D): sums of the per-(batch, tile) partials.  A block covers 32
// outputs (one per lane); warp w sums the partials q = w, w + 8, ... in order, and the 8 warp sums
// are added in warp order: a fixed order, so the result is reproducible.
__global__ void __launch_bounds__(256) conv_bwd_finalize(const ConvParams p, int K) {
  __shared__ float red[8][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + lane;                      // (d, k), k = K for the bias
  const int nout = p.D * (K + 1);
  const int nparts = p.B * p.ntile;
  const size_t stride = (size_t)nout;
  float s = 0.0f;
  if (i < nout) {
    for (int q0 = warp; q0 < nparts; q0 += 8 * 4) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = q0 + 8 * u;
        v[u] = q < nparts ? p.part[(size_t)q * stride + i] : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) s += v[u];
    }
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && i < nout) {
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][lane];
    const int d = i / (K + 1), k = i % (K + 1);
    if (k < K) {
      p.dw[(size_t)d * K + k] = t;
    } else if (p.db != nullptr) {
      p.db[d] = t;
    }
  }
}

int fail(int code, const char* fmt, long long a = 0, long long b = 0) {
  char msg[256];
  snprintf(msg, sizeof(msg), fmt, a, b);
  return ssm::report_error(code, msg);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T, int VEC>
cudaError_t launch_k(bool bwd, int K, const ConvParams& p, cudaStream_t st) {
  const dim3 grid((unsigned)((p.D / VEC + kThreads - 1) / kThreads), (unsigned)p.ntile, (unsigned)p.B);
  switch (K) {
#define SSM_CONV_CASE(KK)                                                                       \
  case KK:                                                                                      \
    if (bwd) conv_bwd_kernel<T, VEC, KK><<<grid, kThreads, 0, st>>>(p);                        \
    else conv_fwd_kernel<T, VEC, KK><<<grid, kThreads, 0, st>>>(p);                            \
    break;
    SSM_CONV_CASE(1)
    SSM_CONV_CASE(2)
    SSM_CONV_CASE(3)
    SSM_CONV_CASE(4)
#undef SSM_CONV_CASE
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// 16-byte vectors when every row start of every view is 16-byte aligned.
cudaError_t launch(bool bwd, int dtype, int K, const ConvParams& p, bool vec, cudaStream_t st) {
  if (dtype == SSM_BF16)
    return vec ? launch_k<__nv_bfloat16, 8>(bwd, K, p, st) : launch_k<__nv_bfloat16, 1>(bwd, K, p, st);
  return vec ? launch_k<float, 4>(bwd, K, p, st) : launch_k<float, 1>(bwd, K, p, st);
}

bool rows_aligned(const ssm_view& v, int esize) {
  return v.ptr == nullptr ||
         (al16(v.ptr) && (v.batch_stride * esize) % 16 == 0 && (v.row_stride * esize) % 16 == 0);
}

int check_shape(int64_t B, int64_t L, int64_t D, int64_t K, const ssm_view& x, const float* w) {
  if (B < 1 || L < 1 || D < 1 || B > 65535 || L > (1LL << 30) || D > (1LL << 24))
    return fail(SSM_ERR_INVALID, "conv1d: shape B=%lld L=%lld out of range", B, L);
  if (K < 1 || K > 4) return fail(SSM_ERR_UNSUPPORTED, "conv1d: kernel width %lld unsupported (1..4)", K);
  if (x.ptr == nullptr || w == nullptr) return fail(SSM_ERR_INVALID, "conv1d: x and weight are required");
  if (x.dtype != SSM_F32 && x.dtype != SSM_BF16) return fail(SSM_ERR_DTYPE, "conv1d: x dtype %lld unsupported", x.dtype);
  if (x.row_stride < 0 || x.batch_stride < 0) return fail(SSM_ERR_INVALID, "conv1d: negative strides");
  return SSM_OK;
}

}  // namespace

extern "C" {

int ssm_conv1d_fwd(int64_t B, int64_t L, int64_t D, int64_t K, ssm_view x, const float* weight, const float* bias,
                   const void* conv_state, int32_t silu, ssm_view out, void* new_conv_state, void* stream) {
  int rc = check_shape(B, L, D, K, x, weight);
  if (rc) return rc;
  if (out.ptr == nullptr || out.dtype != x.dtype) return fail(SSM_ERR_DTYPE, "conv1d: out must be given in x's dtype");
  const int es = x.dtype == SSM_BF16 ? 2 : 4;
  const int vecw = 16 / es;
  const bool vec = D % vecw == 0 && rows_aligned(x, es) && rows_aligned(out, es);
  const int tt = tile_len(B, L, D, vec ? vecw : 1);
  if (new_conv_state != nullptr && new_conv_state == conv_state && L > tt)
    return fail(SSM_ERR_INVALID, "conv1d: in-place state update needs a single time tile (L <= %lld, got L=%lld)",
                tt, L);
  ConvParams p = {};
  p.x = x.ptr;
  p.xsb = x.batch_stride;
  p.xsl = x.row_stride;
  p.out = const_cast<void*>(out.ptr);
  p.osb = out.batch_stride;
  p.osl = out.row_stride;
  p.w = weight;
  p.bias = bias;
  p.state = conv_state;
  p.new_state = new_conv_state;
  p.B = (int)B;
  p.L = (int)L;
  p.D = (int)D;
  p.tt = tt;
  p.ntile = (int)((L + tt - 1) / tt);
  p.silu = silu ? 1 : 0;
  cudaError_t e = launch(false, x.dtype, (int)K, p, vec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(SSM_ERR_CUDA, "conv1d forward launch failed (error %lld)", (long long)e);
  return SSM_OK;
}

int ssm_conv1d_bwd_workspace_size(int64_t B, int64_t L, int64_t D, int64_t K, size_t* bytes) {
  if (bytes == nullptr) return fail(SSM_ERR_INVALID, "conv1d: bytes is NULL");
  if (B < 1 || L < 1 || D < 1 || K < 1 || K > 4) return fail(SSM_ERR_INVALID, "conv1d: bad shape B=%lld L=%lld", B, L);
  // sized for the shortest tile any dtype / alignment could choose
  *bytes = (size_t)B * ((L + 3) / 4) * D * (K + 1) * sizeof(float);
  return SSM_OK;
}

int ssm_conv1d_bwd(int64_t B, int64_t L, int64_t D, int64_t K, ssm_view x, const float* weight, const float* bias,
                   int32_t silu, ssm_view dout, ssm_view dx, float* dweight, float* dbias, void* workspace,
                   size_t workspace_bytes, void* stream) {
  int rc = check_shape(B, L, D, K, x, weight);
  if (rc) return rc;
  if (dout.ptr == nullptr || dout.dtype != x.dtype || dx.ptr == nullptr || dx.dtype != x.dtype)
    return fail(SSM_ERR_DTYPE, "conv1d: dout and dx must be given in x's dtype");
  if (dweight == nullptr) return fail(SSM_ERR_INVALID, "conv1d: dweight is required");
  size_t need = 0;
  ssm_conv1d_bwd_workspace_size(B, L, D, K, &need);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(SSM_ERR_WORKSPACE, "conv1d backward workspace of %lld bytes required, %lld given", (long long)need,
                (long long)workspace_bytes);
  const int es = x.dtype == SSM_BF16 ? 2 : 4;
  const int vecw = 16 / es;
  const bool vec = D % vecw == 0 && rows_aligned(x, es) && rows_aligned(dout, es) && rows_aligned(dx, es);
  const int tt = tile_len(B, L, D, vec ? vecw : 1);
  ConvParams p = {};
  p.x = x.ptr;
  p.xsb = x.batch_stride;
  p.xsl = x.row_stride;
  p.out = const_cast<void*>(dx.ptr);
  p.osb = dx.batch_stride;
  p.osl = dx.row_stride;
  p.dout = dout.ptr;
  p.gsb = dout.batch_stride;
  p.gsl = dout.row_stride;
  p.w = weight;
  p.bias = bias;
  p.part = static_cast<float*>(workspace);
  p.dw = dweight;
  p.db = dbias;
  p.B = (int)B;
  p.L = (int)L;
  p.D = (int)D;
  p.tt = tt;
  p.ntile = (int)((L + tt - 1) / tt);
  p.silu = silu ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch(true, x.dtype, (int)K, p, vec, st);
  if (e != cudaSuccess) return fail(SSM_ERR_CUDA, "conv1d backward launch failed (error %lld)", (long long)e);
  const int n = (int)(D * (K + 1));
  conv_bwd_finalize<<<(n + 31) / 32, 256, 0, st>>>(p, (int)K);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SSM_ERR_CUDA, "conv1d finalize launch failed (error %lld)", (long long)e);
  return SSM_OK;
}

}  // extern "C"
