// ssm_api.cu — the extern "C" entry points declared in include/ssm_b200.h.
//
// Host-side responsibilities: validate shapes / dtypes / alignment, decide whether the
// sequence is split across CTAs, build TMA tensor maps (cuTensorMapEncodeTiled through the
// runtime's driver entry point), carve the caller's workspace and enqueue the kernels on the
// caller's stream.  Nothing here allocates device memory or synchronises, so every entry
// point except ssm_read_device_error can be captured in a CUDA graph.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "ssm_b200.h"
#include "ssm_bwd.cuh"
#include "ssm_fwd.cuh"

namespace ssm {
cudaError_t launch_carry(const CarryParams& p, cudaStream_t stream);
cudaError_t launch_compose(const float* decay, const float* end, const float* start, float* out, float* last, int W,
                           long long elems, long long stride, int reverse, cudaStream_t stream);
cudaError_t launch_update(int N, bool bf16, const UpdParams& p, cudaStream_t stream);
}  // namespace ssm

using namespace ssm;

namespace ssm {
// Internal (not exported): lets other translation units set the message ssm_last_error_message
// returns.
int report_error(int code, const char* msg);
}  // namespace ssm

// Device-side error word set by kernels whose bounded waits gave up.
__device__ int g_ssm_device_error = 0;

namespace {

thread_local char g_msg[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SSM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int* device_error_ptr() {
  static std::mutex mu;
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_ssm_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool valid_n(int64_t N) { return N == 4 || N == 8 || N == 16 || N == 32 || N == 64; }
bool valid_method(int32_t m) { return m == SSM_ZOH || m == SSM_EULER || m == SSM_BILINEAR; }
size_t esize(int dtype) { return dtype == SSM_BF16 ? 2 : 4; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

DAct dact(const ssm_view& v) {
  DAct a;
  a.ptr = v.ptr;
  a.sb = v.batch_stride;
  a.sl = v.row_stride;
  return a;
}

// Can TMA describe this (B, rows, cols) view?  16-byte aligned base and strides.
bool tma_ok(const ssm_view& v, int64_t B, int64_t rows, int64_t cols) {
  const size_t e = esize(v.dtype);
  if (!aligned16(v.ptr)) return false;
  if (rows > 1 && ((v.row_stride * (int64_t)e) % 16 != 0 || v.row_stride < cols)) return false;
  if (B > 1 && ((v.batch_stride * (int64_t)e) % 16 != 0 || v.batch_stride < cols)) return false;
  return true;
}

// 3-D tensor map over a (B, rows, cols) view with a (box_cols x box_rows x 1) box.
bool make_map(CUtensorMap* m, const ssm_view& v, int64_t B, int64_t rows, int64_t cols, int box_cols,
              int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  const size_t e = esize(v.dtype);
  // strides of unit-extent dimensions do not address memory; give them any legal value
  int64_t sl = v.row_stride, sb = v.batch_stride;
  if (rows <= 1) sl = ((cols * (int64_t)e + 15) / 16) * 16 / (int64_t)e;
  if (B <= 1) sb = sl * std::max<int64_t>(rows, 1);
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)(sl * (int64_t)e), (cuuint64_t)(sb * (int64_t)e)};
  cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, v.dtype == SSM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                   const_cast<void*>(v.ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

// States per thread.  G = 4 is the default: with fewer states per thread the shared-memory
// traffic per element (B, C and the per-channel inputs are re-read by every lane) and the
// reduction work grow faster than the extra warps help, which measurements on B200 confirmed
// for every shape tried.  G = 2 is built for N = 8 and 16; SSM_B200_STATES_PER_THREAD=2|4
// overrides the choice (tuning, tests).
int choose_g(int64_t B, int64_t D, int64_t N) {
  (void)B;
  (void)D;
  if (N != 8 && N != 16) return 4;
  if (const char* env = getenv("SSM_B200_STATES_PER_THREAD")) {
    if (env[0] == '2') return 2;
  }
  return 4;
}

// Sequence split of the forward: S segments of seg_len steps (a multiple of 16).  The forward runs one warp per (batch, CPW channels); when that
// is fewer than two warps per SM (long sequences over few channels: B = 1, D = 512 gives 64
// warps) the sequence is cut into S segments of at least 8 chunks, aiming at 64 warps' worth of
// work per SM (several waves: shorter segments balance better).  A split costs one extra pass
// without outputs (measured on config-1 shapes: S = 2 is 35 % slower than S = 1), so shapes with
// enough warps are not split.  (B = 1, L = 131072, D = 512: S = 148 takes 0.90 ms, S = 19 1.28 ms.)
void plan_segments(int64_t B, int64_t L, int64_t D, int64_t N, int* nseg, int* seg_len) {
  const int64_t cpw = 32 * choose_g(B, D, N) / N;
  const int64_t warps = B * ((D + cpw - 1) / cpw);
  const int64_t nchunk = (L + kChunk - 1) / kChunk;
  const int64_t sms = sm_count();
  int64_t S = 1;
  if (warps < 2 * sms && nchunk >= 16) S = std::min<int64_t>((64 * sms + warps - 1) / warps, nchunk / 8);
  if (const char* env = getenv("SSM_B200_FWD_SEGMENTS")) {   // override, for measurements
    const long v = strtol(env, nullptr, 10);
    if (v >= 1) S = std::min<int64_t>(v, nchunk);
  }
  if (S < 1) S = 1;
  int64_t len = ((L + S - 1) / S + kChunk - 1) / kChunk * kChunk;
  S = (L + len - 1) / len;
  *nseg = (int)S;
  *seg_len = (int)len;
}

// Sequence split of the backward.  One CTA per (batch, 32 channels) walks the whole sequence; when
// those CTAs fill at most 3/4 of the slots the GPU has for them (B = 1, D = 512: 16 CTAs; config 3
// sharded over 8 GPUs: 160, over 4: 320 of 444), the sequence is cut into S segments, one CTA each: enough to fill the
// slots once, and segments of at most 16 chunks (256 steps; more, shorter segments balance better),
// but at least 8 chunks each.  Measured on one B200 (backward ms, S): B=1 L=4096 D=512 fp32 0.819 (1),
// 0.166 (8), 0.109 (18), 0.114 (32); B=4 L=4096 D=512 fp32 0.794 (1), 0.371 (4), 0.332 (16);
// B=8 L=8192 D=640 bf16 2.25 (1), 1.62 (5), 1.50 (8), 1.48 (16), 1.47 (24); B=8 L=8192 D=1280 bf16
// 3.21 (1), 2.82 (16); config 1 (256 CTAs of 296 slots) 0.146 (1), 0.174 (2): not split.  The split costs the
// adjoint summaries of segments 1 .. S-1 (the forward kernel's adjoint mode) and a reverse carry.
int64_t bwd_ctas_per_sm(int64_t N, int dtype) {
  switch (N) {
    case 4: return 8;
    case 8: return 4;
    case 16: return dtype == SSM_BF16 ? 3 : 2;
    default: return 1;
  }
}
void plan_bwd_segments(int64_t B, int64_t L, int64_t D, int64_t N, int dtype, int* nseg, int* seg_len) {
  const int64_t ctas = B * ((D + 31) / 32);
  const int64_t slots = bwd_ctas_per_sm(N, dtype) * sm_count();
  const int64_t nchunk = (L + kChunk - 1) / kChunk;
  int64_t S = 1;
  if (4 * ctas <= 3 * slots && nchunk >= 16) S = std::min<int64_t>(std::max<int64_t>(slots / ctas, nchunk / 16), nchunk / 8);
  if (const char* env = getenv("SSM_B200_BWD_SEGMENTS")) {   // override, for measurements
    const long v = strtol(env, nullptr, 10);
    if (v >= 1) S = std::min<int64_t>(v, nchunk);
  }
  if (S < 1) S = 1;
  int64_t len = ((L + S - 1) / S + kChunk - 1) / kChunk * kChunk;
  S = (L + len - 1) / len;
  *nseg = (int)S;
  *seg_len = (int)len;
}

// Workspace arrays are carved at 256-byte boundaries (carve below): a size counts the alignment of the
// base pointer and every array rounded up.
size_t carved(size_t nfloat) { return (nfloat * sizeof(float) + 255) / 256 * 256; }
size_t seg_ws_bytes(int64_t B, int64_t S, int64_t D, int64_t N) { return 256 + 3 * carved((size_t)B * S * D * N); }

size_t fwd_ws_bytes(int64_t B, int64_t L, int64_t D, int64_t N) {
  int S, len;
  plan_segments(B, L, D, N, &S, &len);
  if (S <= 1) return 0;
  return seg_ws_bytes(B, S, D, N);
}

// Workspace of a backward with S segments: the dB | dC partials, the (batch, segment) partials of
// dA, dD and d(bias), and for S > 1 the incoming adjoints and the adjoint pass's three segment
// arrays (decay, adjoint from zero, carry).
size_t bwd_ws_bytes_for(int64_t B, int64_t L, int64_t D, int64_t N, int64_t S) {
  const int64_t ndt = (D + 31) / 32;
  const size_t own = 256 + carved((size_t)B * ndt * L * 2 * N) + carved((size_t)B * S * D * N) +
                     2 * carved((size_t)B * S * D);
  const size_t segs = S > 1 ? carved((size_t)B * S * D * N) + seg_ws_bytes(B, S, D, N) : 0;
  return own + segs;
}
// the size the API reports: enough for either element type's segment plan
size_t bwd_ws_bytes(int64_t B, int64_t L, int64_t D, int64_t N) {
  size_t need = 0;
  for (int dtype : {SSM_F32, SSM_BF16}) {
    int S, len;
    plan_bwd_segments(B, L, D, N, dtype, &S, &len);
    need = std::max(need, bwd_ws_bytes_for(B, L, D, N, S));
  }
  return need;
}

float* carve(unsigned char*& cur, size_t nfloat) {
  float* p = reinterpret_cast<float*>(cur);
  cur += (nfloat * sizeof(float) + 255) / 256 * 256;
  return p;
}

int check_common(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method) {
  if (B < 1 || L < 1 || D < 1) return fail(SSM_ERR_INVALID, "shape B=%lld L=%lld D=%lld must be positive",
                                           (long long)B, (long long)L, (long long)D);
  if (B > 65535) return fail(SSM_ERR_INVALID, "batch %lld exceeds 65535", (long long)B);
  if (L > (int64_t)1 << 30 || D > (int64_t)1 << 24)
    return fail(SSM_ERR_INVALID, "L=%lld / D=%lld too large", (long long)L, (long long)D);
  if (!valid_n(N))
    return fail(SSM_ERR_INVALID, "d_state N=%lld unsupported: must be one of 4, 8, 16, 32, 64", (long long)N);
  if (!valid_method(method)) return fail(SSM_ERR_INVALID, "unknown discretization method %d", (int)method);
  return SSM_OK;
}

int check_view(const char* name, const ssm_view& v, int dtype, int64_t cols, bool required) {
  if (v.ptr == nullptr) return required ? fail(SSM_ERR_INVALID, "%s is required", name) : SSM_OK;
  if (v.dtype != dtype)
    return fail(SSM_ERR_DTYPE, "%s dtype %d differs from u's dtype %d (upcast mixed inputs first)", name,
                (int)v.dtype, dtype);
  if (v.row_stride < 0 || v.batch_stride < 0) return fail(SSM_ERR_INVALID, "%s has negative strides", name);
  (void)cols;
  return SSM_OK;
}

int check_f32(const char* name, const void* p, bool required) {
  if (p == nullptr) return required ? fail(SSM_ERR_INVALID, "%s is required", name) : SSM_OK;
  if (!aligned16(p)) return fail(SSM_ERR_INVALID, "%s must be 16-byte aligned", name);
  return SSM_OK;
}

// Shared body of ssm_scan_fwd / ssm_scan_fwd_finish / ssm_scan_fwd_summary.
// phase: 0 = full forward, 1 = summary only (writes decay/hend), 2 = finish (reuses the
// per-segment summaries a phase-1 call left in the workspace), 3 = adjoint summary (u carries
// dy and Bm carries C; writes decay and the adjoint at the sequence start into decay/hend),
// 4 = the backward's segment adjoints: the adjoint summaries of the given plan_S segments of plan_len
// steps composed in reverse from h0 (dlast), the adjoint entering every segment written to seg_out.
int fwd_impl(int phase, int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u, ssm_view delta,
             const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z, const float* h0,
             ssm_view y, ssm_view ygate, float* last, float* chunk_states, float* tot_decay, float* tot_hend,
             void* workspace, size_t workspace_bytes, void* stream_v, const ssm_delta_opts* opts = nullptr,
             int plan_S = 0, int plan_len = 0, float* seg_out = nullptr) {
  int rc = check_common(B, L, D, N, method);
  if (rc) return rc;
  if (u.ptr == nullptr) return fail(SSM_ERR_INVALID, "u is required");
  const int dt = u.dtype;
  if (dt != SSM_F32 && dt != SSM_BF16) return fail(SSM_ERR_DTYPE, "u dtype %d unsupported", dt);
  if ((rc = check_view("delta", delta, dt, D, true))) return rc;
  if ((rc = check_view("Bm", Bm, dt, N, true))) return rc;
  const bool summary = (phase == 1 || phase == 3 || phase == 4);
  const bool adjoint = (phase == 3 || phase == 4);
  if (adjoint && (rc = check_view("z", z, dt, D, false))) return rc;
  if (!summary) {
    if ((rc = check_view("Cm", Cm, dt, N, true))) return rc;
    if ((rc = check_view("z", z, dt, D, false))) return rc;
    if ((rc = check_view("y", y, dt, D, true))) return rc;
    if ((rc = check_view("ygate", ygate, dt, D, false))) return rc;
  }
  if ((rc = check_f32("A", A, true))) return rc;
  if ((rc = check_f32("Dskip", Dskip, false))) return rc;
  if ((rc = check_f32("h0", h0, false))) return rc;
  if ((rc = check_f32("last", last, false))) return rc;
  if ((rc = check_f32("chunk_states", chunk_states, false))) return rc;
  if ((phase == 1 || phase == 3) &&
      (tot_decay == nullptr || tot_hend == nullptr || !aligned16(tot_decay) || !aligned16(tot_hend)))
    return fail(SSM_ERR_INVALID, "the two summary outputs are required and must be 16-byte aligned");
  if (phase == 4 && (plan_S < 2 || seg_out == nullptr)) return fail(SSM_ERR_INVALID, "segment adjoints need S > 1");
  const size_t need = phase == 4 ? seg_ws_bytes(B, plan_S, D, N) : fwd_ws_bytes(B, L, D, N);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(SSM_ERR_WORKSPACE, "forward workspace of %zu bytes required, %zu given", need, workspace_bytes);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);

  FwdParams p;
  memset(&p, 0, sizeof(p));
  p.u = dact(u);
  p.dt = dact(delta);
  p.z = dact(z);
  p.Bm = dact(Bm);
  p.Cm = dact(Cm);
  p.y = dact(y);
  p.yg = dact(ygate);
  p.save_ygate = (!summary && ygate.ptr != nullptr) ? 1 : 0;
  p.A = A;
  p.Dskip = Dskip;
  p.last = last;
  p.chunk_states = chunk_states;
  p.err = device_error_ptr();
  p.B = (int)B;
  p.L = (int)L;
  p.D = (int)D;
  p.nchunks = (int)((L + kChunk - 1) / kChunk);
  p.has_z = z.ptr != nullptr;
  if (opts != nullptr && opts->softplus) {
    if (opts->bias != nullptr && !aligned16(opts->bias)) return fail(SSM_ERR_INVALID, "delta bias must be 16-byte aligned");
    p.dt_softplus = 1;
    p.dt_bias = opts->bias;
  }

  // one warp per CTA: its TMA boxes are CPW channels wide, widened to 16 bytes of channels
  const int G = choose_g(B, D, N);
  const int cpw = (int)(32 * G / N);
  const int bxc = std::max<int>(cpw, (int)(16 / esize(dt)));
  bool use_tma = tma_ok(u, B, L, D) && tma_ok(delta, B, L, D) && tma_ok(Bm, B, L, N);
  if (!summary) use_tma = use_tma && tma_ok(Cm, B, L, N);
  if (phase != 1) use_tma = use_tma && (!p.has_z || tma_ok(z, B, L, D));
  int S, len;
  if (phase == 4) {
    S = plan_S;
    len = plan_len;
  } else {
    plan_segments(B, L, D, N, &S, &len);
  }
  p.nseg = S;
  p.seg_len = len;
  // TMA boxes of kb 16-step tiles: 4 for an unsplit main pass whose warps (one per CTA) all fit on
  // the GPU at once with the larger ring's shared memory, else 2 (split sequences with short
  // segments, summary passes, grids that would need extra waves)
  const bool bf = dt == SSM_BF16;
  const int64_t fwd_warps = B * ((D + cpw - 1) / cpw);
  const int smem4 = bf ? fwd_smem_bytes<__nv_bfloat16>((int)N, G, 4) : fwd_smem_bytes<float>((int)N, G, 4);
  const int64_t ctas4 = std::min<int64_t>(32, (228 * 1024) / (smem4 + 1024));   // per SM
  const int kb = (S == 1 && !summary && fwd_warps <= ctas4 * (int64_t)sm_count()) ? 4 : 2;
  if (use_tma) {
    const int rows = kChunk * kb;
    bool ok = make_map(&p.tm_u, u, B, L, D, bxc, rows) && make_map(&p.tm_dt, delta, B, L, D, bxc, rows) &&
              make_map(&p.tm_B, Bm, B, L, N, (int)N, rows);
    if (!summary) ok = ok && make_map(&p.tm_C, Cm, B, L, N, (int)N, rows);
    if (phase != 1 && p.has_z) ok = ok && make_map(&p.tm_z, z, B, L, D, bxc, rows);
    use_tma = ok;
  }
  p.use_tma = use_tma ? 1 : 0;
  const unsigned ndt = (unsigned)((D + 31) / 32);
  const dim3 grid(ndt, (unsigned)S, (unsigned)B);
  auto launch = [&](int mode, const FwdParams& q) {
    // segments [seg_first, S): the backward's segment adjoints skip segment 0 (nothing precedes it)
    const dim3 g(grid.x, grid.y - (unsigned)q.seg_first, grid.z);
    return bf ? launch_fwd<__nv_bfloat16>((int)N, G, method, mode, kb, q, g, stream)
              : launch_fwd<float>((int)N, G, method, mode, kb, q, g, stream);
  };
  cudaError_t e;

  const int smode = adjoint ? kModeAdjoint : kModeSummary;
  if (S == 1) {
    if (summary) {
      FwdParams q = p;
      q.seg_hend = tot_hend;
      q.seg_decay = tot_decay;
      if ((e = launch(smode, q)) != cudaSuccess) return cuda_fail(e, "summary launch");
      return SSM_OK;
    }
    p.h_init = h0;
    if ((e = launch(kModeMain, p)) != cudaSuccess) return cuda_fail(e, "forward launch");
    return SSM_OK;
  }

  unsigned char* cur = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  const size_t segn = (size_t)B * S * D * N;
  float* seg_hend = carve(cur, segn);
  float* seg_decay = carve(cur, segn);
  float* seg_init = carve(cur, segn);

  if (phase != 2) {
    FwdParams q = p;
    q.seg_hend = seg_hend;
    q.seg_decay = seg_decay;
    q.seg_first = phase == 4 ? 1 : 0;   // the reverse carry never uses segment 0's summary
    if ((e = launch(smode, q)) != cudaSuccess) return cuda_fail(e, "summary launch");
  }
  CarryParams cp;
  memset(&cp, 0, sizeof(cp));
  cp.h_init = (summary && phase != 4) ? nullptr : h0;
  cp.seg_decay = seg_decay;
  cp.seg_hend = seg_hend;
  cp.seg_init = phase == 4 ? seg_out : summary ? nullptr : seg_init;
  cp.tot_decay = (summary && phase != 4) ? tot_decay : nullptr;
  cp.tot_hend = (summary && phase != 4) ? tot_hend : nullptr;
  cp.B = (int)B;
  cp.D = (int)D;
  cp.N = (int)N;
  cp.nseg = S;
  cp.reverse = adjoint ? 1 : 0;
  if ((e = launch_carry(cp, stream)) != cudaSuccess) return cuda_fail(e, "carry launch");
  if (summary) return SSM_OK;
  p.seg_init = seg_init;
  if ((e = launch(kModeMain, p)) != cudaSuccess) return cuda_fail(e, "forward launch");
  return SSM_OK;
}

}  // namespace

int ssm::report_error(int code, const char* msg) { return fail(code, "%s", msg); }

extern "C" {

int ssm_abi_version(void) { return SSM_B200_ABI_VERSION; }

const char* ssm_last_error_message(void) { return g_msg; }

int ssm_read_device_error(int32_t* flags) {
  int* p = device_error_ptr();
  if (p == nullptr) return fail(SSM_ERR_CUDA, "device error word unavailable");
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "reading device error word");
  const int zero = 0;
  e = cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "clearing device error word");
  if (flags) *flags = v;
  return SSM_OK;
}

int ssm_scan_fwd_workspace_size(int64_t B, int64_t L, int64_t D, int64_t N, size_t* bytes) {
  if (bytes == nullptr) return fail(SSM_ERR_INVALID, "bytes is NULL");
  int rc = check_common(B, L, D, N, SSM_ZOH);
  if (rc) return rc;
  *bytes = fwd_ws_bytes(B, L, D, N);
  return SSM_OK;
}

int ssm_scan_bwd_workspace_size(int64_t B, int64_t L, int64_t D, int64_t N, size_t* bytes) {
  if (bytes == nullptr) return fail(SSM_ERR_INVALID, "bytes is NULL");
  int rc = check_common(B, L, D, N, SSM_ZOH);
  if (rc) return rc;
  *bytes = bwd_ws_bytes(B, L, D, N);
  return SSM_OK;
}

int ssm_compose_shards(int32_t W, int64_t B, int64_t D, int64_t N, const float* decay, const float* end,
                       int64_t shard_stride, const float* start, int32_t reverse, float* out, float* last,
                       void* stream) {
  const int64_t elems = B * D * N;
  if (shard_stride == 0) shard_stride = elems;
  if (shard_stride < elems) return fail(SSM_ERR_INVALID, "shard_stride %lld is below B*D*N", (long long)shard_stride);
  if (W < 1 || B < 1 || D < 1 || N < 1)
    return fail(SSM_ERR_INVALID, "shape W=%d B=%lld D=%lld N=%lld must be positive", (int)W, (long long)B,
                (long long)D, (long long)N);
  if (decay == nullptr || end == nullptr || out == nullptr)
    return fail(SSM_ERR_INVALID, "decay, end and out are required");
  cudaError_t e = launch_compose(decay, end, start, out, last, (int)W, (long long)elems, (long long)shard_stride,
                                 reverse ? 1 : 0, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "compose launch");
  return SSM_OK;
}

int ssm_scan_bwd_plan(int64_t B, int64_t L, int64_t D, int64_t N, int32_t dtype, int32_t* nseg, int32_t* seg_len) {
  if (nseg == nullptr || seg_len == nullptr) return fail(SSM_ERR_INVALID, "nseg and seg_len are required");
  int rc = check_common(B, L, D, N, SSM_ZOH);
  if (rc) return rc;
  if (dtype != SSM_F32 && dtype != SSM_BF16) return fail(SSM_ERR_DTYPE, "dtype %d unsupported", (int)dtype);
  int S, len;
  plan_bwd_segments(B, L, D, N, dtype, &S, &len);
  *nseg = S;
  *seg_len = len;
  return SSM_OK;
}

int ssm_scan_fwd(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u, ssm_view delta,
                 const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z, const float* h0,
                 ssm_view y, ssm_view ygate, float* last, float* chunk_states, void* workspace,
                 size_t workspace_bytes, void* stream) {
  return fwd_impl(0, B, L, D, N, method, u, delta, A, Bm, Cm, Dskip, z, h0, y, ygate, last, chunk_states, nullptr,
                  nullptr, workspace, workspace_bytes, stream);
}

int ssm_scan_fwd_summary(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u, ssm_view delta,
                         const float* A, ssm_view Bm, float* decay, float* hend, void* workspace,
                         size_t workspace_bytes, void* stream) {
  ssm_view none;
  memset(&none, 0, sizeof(none));
  none.dtype = u.dtype;
  return fwd_impl(1, B, L, D, N, method, u, delta, A, Bm, none, nullptr, none, nullptr, none, none, nullptr,
                  nullptr, decay, hend, workspace, workspace_bytes, stream);
}

int selective_scan_fwd(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u, ssm_view delta,
                       const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z, const float* h0,
                       ssm_view y, ssm_view ygate, float* last, float* chunk_states, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return ssm_scan_fwd(B, L, D, N, method, u, delta, A, Bm, Cm, Dskip, z, h0, y, ygate, last, chunk_states,
                      workspace, workspace_bytes, stream);
}

int selective_scan_bwd(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u, ssm_view delta,
                       const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z, const float* h0,
                       const float* chunk_states, ssm_view ygate, ssm_view dy, const float* dlast, ssm_view du,
                       ssm_view ddelta, float* dA, ssm_view dBm, ssm_view dCm, float* dDskip, ssm_view dz,
                       float* dh0, void* workspace, size_t workspace_bytes, void* stream) {
  return ssm_scan_bwd(B, L, D, N, method, u, delta, A, Bm, Cm, Dskip, z, h0, chunk_states, ygate, dy, dlast, du,
                      ddelta, dA, dBm, dCm, dDskip, dz, dh0, workspace, workspace_bytes, stream);
}

int selective_state_update(int64_t B, int64_t D, int64_t N, int32_t method, float* state, ssm_view x,
                           ssm_view delta, const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z,
                           ssm_view y, void* stream) {
  return ssm_state_update(B, D, N, method, state, x, delta, A, Bm, Cm, Dskip, z, y, stream);
}

int ssm_scan_bwd_summary(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view delta,
                         const float* A, ssm_view Cm, ssm_view z, ssm_view dy, float* decay, float* dstart,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (dy.ptr == nullptr) return fail(SSM_ERR_INVALID, "dy is required");
  ssm_view none;
  memset(&none, 0, sizeof(none));
  none.dtype = dy.dtype;
  return fwd_impl(3, B, L, D, N, method, dy, delta, A, Cm, none, nullptr, z, nullptr, none, none, nullptr,
                  nullptr, decay, dstart, workspace, workspace_bytes, stream);
}

int ssm_scan_fwd_finish(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u, ssm_view delta,
                        const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z,
                        const float* h_in, ssm_view y, ssm_view ygate, float* last, float* chunk_states,
                        void* workspace, size_t workspace_bytes, void* stream) {
  return fwd_impl(2, B, L, D, N, method, u, delta, A, Bm, Cm, Dskip, z, h_in, y, ygate, last, chunk_states,
                  nullptr, nullptr, workspace, workspace_bytes, stream);
}

int ssm_scan_bwd(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u, ssm_view delta,
                 const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z, const float* h0,
                 const float* chunk_states, ssm_view ygate, ssm_view dy, const float* dlast, ssm_view du,
                 ssm_view ddelta,
                 float* dA, ssm_view dBm, ssm_view dCm, float* dDskip, ssm_view dz, float* dh0, void* workspace,
                 size_t workspace_bytes, void* stream_v) {
  return ssm_scan_bwd_ex(B, L, D, N, method, u, delta, A, Bm, Cm, Dskip, z, h0, chunk_states, ygate, dy, dlast, du,
                         ddelta, dA, dBm, dCm, dDskip, dz, dh0, nullptr, workspace, workspace_bytes, stream_v);
}

int ssm_scan_fwd_ex(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u, ssm_view delta,
                    const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z, const float* h0,
                    ssm_view y, ssm_view ygate, float* last, float* chunk_states, const ssm_delta_opts* opts,
                    void* workspace, size_t workspace_bytes, void* stream) {
  return fwd_impl(0, B, L, D, N, method, u, delta, A, Bm, Cm, Dskip, z, h0, y, ygate, last, chunk_states, nullptr,
                  nullptr, workspace, workspace_bytes, stream, opts);
}

int ssm_scan_bwd_ex(int64_t B, int64_t L, int64_t D, int64_t N, int32_t method, ssm_view u, ssm_view delta,
                    const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z, const float* h0,
                    const float* chunk_states, ssm_view ygate, ssm_view dy, const float* dlast, ssm_view du,
                    ssm_view ddelta, float* dA, ssm_view dBm, ssm_view dCm, float* dDskip, ssm_view dz, float* dh0,
                    const ssm_delta_opts* opts, void* workspace, size_t workspace_bytes, void* stream_v) {
  int rc = check_common(B, L, D, N, method);
  if (rc) return rc;
  if (u.ptr == nullptr) return fail(SSM_ERR_INVALID, "u is required");
  const int dt = u.dtype;
  if (dt != SSM_F32 && dt != SSM_BF16) return fail(SSM_ERR_DTYPE, "u dtype %d unsupported", dt);
  const bool has_z = z.ptr != nullptr;
  if ((rc = check_view("delta", delta, dt, D, true))) return rc;
  if ((rc = check_view("Bm", Bm, dt, N, true))) return rc;
  if ((rc = check_view("Cm", Cm, dt, N, true))) return rc;
  if ((rc = check_view("z", z, dt, D, false))) return rc;
  if ((rc = check_view("dy", dy, dt, D, true))) return rc;
  if ((rc = check_view("ygate", ygate, dt, D, has_z))) return rc;
  if ((rc = check_view("du", du, dt, D, true))) return rc;
  if ((rc = check_view("ddelta", ddelta, dt, D, true))) return rc;
  if ((rc = check_view("dBm", dBm, dt, N, true))) return rc;
  if ((rc = check_view("dCm", dCm, dt, N, true))) return rc;
  if ((rc = check_view("dz", dz, dt, D, has_z))) return rc;
  if ((rc = check_f32("A", A, true))) return rc;
  if ((rc = check_f32("Dskip", Dskip, false))) return rc;
  if ((rc = check_f32("h0", h0, false))) return rc;
  if ((rc = check_f32("chunk_states", chunk_states, true))) return rc;
  if ((rc = check_f32("dlast", dlast, false))) return rc;
  if ((rc = check_f32("dA", dA, true))) return rc;
  if ((rc = check_f32("dDskip", dDskip, Dskip != nullptr))) return rc;
  if ((rc = check_f32("dh0", dh0, h0 != nullptr))) return rc;
  int S, seg_len;
  plan_bwd_segments(B, L, D, N, dt, &S, &seg_len);
  const size_t need = bwd_ws_bytes_for(B, L, D, N, S);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(SSM_ERR_WORKSPACE, "backward workspace of %zu bytes required, %zu given", need, workspace_bytes);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);

  const int ndt = (int)((D + 31) / 32);
  BwdParams p;
  memset(&p, 0, sizeof(p));
  p.u = dact(u);
  p.dt = dact(delta);
  p.z = dact(z);
  p.dy = dact(dy);
  p.yg = dact(ygate);
  p.Bm = dact(Bm);
  p.Cm = dact(Cm);
  p.du = dact(du);
  p.ddt = dact(ddelta);
  p.dz = dact(dz);
  p.A = A;
  p.Dskip = Dskip;
  p.h0 = h0;
  p.chunk_states = chunk_states;
  p.dlast = dlast;
  p.dh0 = h0 != nullptr ? dh0 : nullptr;
  p.err = device_error_ptr();
  p.B = (int)B;
  p.L = (int)L;
  p.D = (int)D;
  p.nchunks = (int)((L + kChunk - 1) / kChunk);
  p.ndt = ndt;
  p.has_z = has_z ? 1 : 0;
  unsigned char* cur = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  p.part_bc = carve(cur, (size_t)B * ndt * L * 2 * N);
  p.part_A = carve(cur, (size_t)B * S * D * N);
  p.part_D = carve(cur, (size_t)B * S * D);
  p.part_dtb = carve(cur, (size_t)B * S * D);
  p.nseg = S;
  p.seg_len = seg_len;
  if (opts != nullptr && opts->softplus) {
    if (opts->bias != nullptr && !aligned16(opts->bias)) return fail(SSM_ERR_INVALID, "delta bias must be 16-byte aligned");
    p.dt_softplus = 1;
    p.dt_bias = opts->bias;
  }
  if (S > 1) {   // the adjoint entering every segment: summaries of the later segments, composed in reverse
    float* seg_dh = carve(cur, (size_t)B * S * D * N);
    const size_t used = (size_t)(cur - static_cast<unsigned char*>(workspace));
    ssm_view none;
    memset(&none, 0, sizeof(none));
    none.dtype = dt;
    rc = fwd_impl(4, B, L, D, N, method, dy, delta, A, Cm, none, nullptr, z, dlast, none, none, nullptr, nullptr,
                  nullptr, nullptr, cur, workspace_bytes - used, stream_v, opts, S, seg_len, seg_dh);
    if (rc) return rc;
    p.seg_dh = seg_dh;
  }

  bool use_tma = tma_ok(u, B, L, D) && tma_ok(delta, B, L, D) && tma_ok(dy, B, L, D) && tma_ok(Bm, B, L, N) &&
                 tma_ok(Cm, B, L, N) && (!has_z || (tma_ok(z, B, L, D) && tma_ok(ygate, B, L, D)));
  if (use_tma) {
    bool ok = make_map(&p.tm_u, u, B, L, D, 32, kChunk) && make_map(&p.tm_dt, delta, B, L, D, 32, kChunk) &&
              make_map(&p.tm_dy, dy, B, L, D, 32, kChunk) && make_map(&p.tm_B, Bm, B, L, N, (int)N, kChunk) &&
              make_map(&p.tm_C, Cm, B, L, N, (int)N, kChunk);
    if (has_z) ok = ok && make_map(&p.tm_z, z, B, L, D, 32, kChunk) && make_map(&p.tm_yg, ygate, B, L, D, 32, kChunk);
    use_tma = ok;
  }
  p.use_tma = use_tma ? 1 : 0;

  const bool bf = dt == SSM_BF16;
  const dim3 grid((unsigned)ndt, (unsigned)B, (unsigned)S);
  const int G = choose_g(B, D, N);
  cudaError_t e = bf ? launch_bwd<__nv_bfloat16>((int)N, G, method, p, grid, stream)
                     : launch_bwd<float>((int)N, G, method, p, grid, stream);
  if (e != cudaSuccess) return cuda_fail(e, "backward launch");

  FinParams f;
  memset(&f, 0, sizeof(f));
  f.part_bc = p.part_bc;
  f.part_A = p.part_A;
  f.part_D = p.part_D;
  f.dB = dact(dBm);
  f.dC = dact(dCm);
  f.dA = dA;
  f.dD = Dskip != nullptr ? dDskip : nullptr;
  f.part_dtb = p.part_dtb;
  f.ddt_bias = (p.dt_softplus && opts->dbias != nullptr) ? opts->dbias : nullptr;
  f.B = (int)B;
  f.L = (int)L;
  f.D = (int)D;
  f.N = (int)N;
  f.ndt = ndt;
  f.nsum = (int)(B * S);
  e = bf ? launch_bwd_finalize<__nv_bfloat16>(f, stream) : launch_bwd_finalize<float>(f, stream);
  if (e != cudaSuccess) return cuda_fail(e, "backward finalize launch");
  return SSM_OK;
}

int ssm_state_update(int64_t B, int64_t D, int64_t N, int32_t method, float* state, ssm_view x, ssm_view delta,
                     const float* A, ssm_view Bm, ssm_view Cm, const float* Dskip, ssm_view z, ssm_view y,
                     void* stream) {
  int rc = check_common(B, 1, D, N, method);
  if (rc) return rc;
  if (x.ptr == nullptr) return fail(SSM_ERR_INVALID, "x is required");
  const int dt = x.dtype;
  if (dt != SSM_F32 && dt != SSM_BF16) return fail(SSM_ERR_DTYPE, "x dtype %d unsupported", dt);
  if ((rc = check_view("delta", delta, dt, D, true))) return rc;
  if ((rc = check_view("Bm", Bm, dt, N, true))) return rc;
  if ((rc = check_view("Cm", Cm, dt, N, true))) return rc;
  if ((rc = check_view("z", z, dt, D, false))) return rc;
  if ((rc = check_view("y", y, dt, D, true))) return rc;
  if ((rc = check_f32("state", state, true))) return rc;
  if ((rc = check_f32("A", A, true))) return rc;
  if ((rc = check_f32("Dskip", Dskip, false))) return rc;
  UpdParams p;
  memset(&p, 0, sizeof(p));
  p.state = state;
  p.x = dact(x);
  p.dt = dact(delta);
  p.Bm = dact(Bm);
  p.Cm = dact(Cm);
  p.z = dact(z);
  p.y = dact(y);
  p.A = A;
  p.Dskip = Dskip;
  p.B = (int)B;
  p.D = (int)D;
  p.method = method;
  p.has_z = z.ptr != nullptr;
  cudaError_t e = launch_update((int)N, dt == SSM_BF16, p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "state update launch");
  return SSM_OK;
}

}  // extern "C"
