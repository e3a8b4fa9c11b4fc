// Quantised KV cache kernels: quantise-on-write append (E4M3 / INT8), finite check,
// and decode of the valid prefix.  HBM-bound byte work: one 16-lane group owns one
// (batch, token, head) row of D = 128 bf16 values (16-byte loads, 8-byte stores).
//
// Arithmetic follows the CPU branch of quantize_kv_into
// (hymm/models/dit/modules/int8_kv_cache.py:149-158):
//   peak  = max |x|                       (fp32)
//   s     = peak > 0 ? peak / R : 1       (IEEE fp32 division, R = 127 or 448)
//   y     = x / s                         (IEEE fp32 division, correctly rounded: div_rn_by)
//   INT8: code = clamp(y >= 0 ? floor(y + 0.5) : ceil(y - 0.5), -127, 127)
//   E4M3: code = e4m3_rn(clamp(y, -448, 448))
#include "hyb_common.cuh"

namespace hyb {
namespace {

constexpr int kRowLanes = 8;  // lanes per row: 8 x 16 bf16 = 128 values

struct AppendParams {
  int fmt;
  int L, L2, H;  // rows [0, L) from src, [L, L + L2) from src2; the batch index is blockIdx.y
  long long start;
  const __nv_bfloat16* src[2];
  long long s_b[2], s_t[2], s_h[2];
  const __nv_bfloat16* src2[2];
  long long s2_b[2], s2_t[2], s2_h[2];
  void* dst[2];
  long long d_b, d_t, d_h;
  float* scale[2];
  long long c_b, c_t, c_h;
  int* status;
  int step_t, step_h;  // the grid stride (groups) split as step_t * H + step_h
};

__device__ __forceinline__ void unpack8(const uint4& u, float* x) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(p[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// max(|a|, |b|, |c|), NaN if any operand is NaN (so a row's non-finite values survive the
// reduction and are caught from the peak alone).
__device__ __forceinline__ float absmax3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(fabsf(a)), "f"(fabsf(b)), "f"(fabsf(c)));
  return r;
}
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// RN(p / R) for R = 127 or 448 from RN(1 / R) by two residual corrections (the division
// scheme named at div_rn_by2 below, with a constant divisor).  Checked against IEEE division
// for every positive finite bf16 p, subnormal quotients included, which covers every row peak.
template <int FMT>
__device__ __forceinline__ float row_scale(float peak) {
  constexpr float R = FMT == HYB_FMT_INT8 ? 127.0f : 448.0f;
  constexpr float rR = FMT == HYB_FMT_INT8 ? 0x1.020408p-7f : 0x1.24924ap-9f;  // RN(1 / R)
  const float q0 = __fmul_rn(peak, rR);
  const float q1 = __fmaf_rn(__fmaf_rn(-R, q0, peak), rR, q0);
  return __fmaf_rn(__fmaf_rn(-R, q1, peak), rR, q1);
}

// x / s rounded to nearest for a pair, from r = RN(1/s): q0 = RN(x r), then two residual steps
// q' = RN(q + r (x - s q)) with the residual formed exactly by the fma.  The first step leaves
// q1 within one ulp of x / s; correcting a quotient that close with a correctly rounded
// reciprocal gives RN(x / s) (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Develop. 34(1), 1990; restated in Muller et al.,
// Handbook of Floating-Point Arithmetic, on FMA-based division).  Valid for every x of a row
// whose scale s is at least 2^-90: the residuals stay normal unless |x| < 2^-103, and such an x
// has |x / s| < 2^-13, whose e4m3 and INT8 codes are 0 whatever the last bit of the quotient.
// The sign of a zero quotient is not kept (x = -0 gives +0): the E4M3 caller restores it on the
// codes, and INT8 has no negative zero.
__device__ __forceinline__ float2 div_rn_by2(float2 x, float s, float r) {
  const float2 rr = make_float2(r, r);
  const float2 ns = make_float2(-s, -s);
  const float2 q0 = fmul2(x, rr);
  const float2 q1 = ffma2(ffma2(ns, q0, x), rr, q0);
  return ffma2(ffma2(ns, q1, x), rr, q1);
}

// Codes of 4 values (one 32-bit word, value i in byte i) from their quotients.
template <int FMT>
__device__ __forceinline__ uint32_t codes4(float2 ya, float2 yb, uint32_t wa, uint32_t wb) {
  if constexpr (FMT == HYB_FMT_INT8) {
    // y >= 0 ? floor(RN(y + 0.5)) : ceil(RN(y - 0.5)) is trunc(RN(y + copysign(0.5, y))); with
    // |y| <= 127 (1 + 2^-23) it lies in [-127, 127], so the reference's clamp never binds.
    const float y[4] = {ya.x, ya.y, yb.x, yb.y};
    uint32_t c[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      c[i] = static_cast<uint32_t>(__float2int_rz(__fadd_rn(y[i], copysignf(0.5f, y[i]))));
    return __byte_perm(__byte_perm(c[0], c[1], 0x0040), __byte_perm(c[2], c[3], 0x0040), 0x5410);
  } else {
    // |y| <= 448 up to rounding; the saturating conversion maps anything beyond to +-448
    // exactly as the reference's clamp does.  The sign bits of the four bf16 inputs (their
    // high bytes) are ORed in: a no-op except for x = -0, whose code is 0x80 (-0 / s = -0).
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(ya, __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(yb, __NV_SATFINITE, __NV_E4M3);
    return (lo | (hi << 16)) | (__byte_perm(wa, wb, 0x7531) & 0x80808080u);
  }
}

// Quantise one 128-value row held by an 8-lane group (16 values per lane: raw[0] holds values
// [8 l, 8 l + 8), raw[1] values [64 + 8 l, 72 + 8 l) of lane l).  Returns the row scale and
// this lane's 16 code bytes in the same two halves.
template <int FMT>
__device__ __forceinline__ float quantise_row16(const uint4 (&raw)[2], unsigned gmask, uint2 (&codes)[2],
                                                bool& nonfinite) {
  float x[16];
  unpack8(raw[0], x);
  unpack8(raw[1], x + 8);
  float peak = absmax3_nan(x[0], x[1], x[2]);
  peak = max_nan(peak, absmax3_nan(x[3], x[4], x[5]));
  peak = max_nan(peak, absmax3_nan(x[6], x[7], x[8]));
  peak = max_nan(peak, absmax3_nan(x[9], x[10], x[11]));
  peak = max_nan(peak, absmax3_nan(x[12], x[13], x[14]));
  peak = max_nan(peak, fabsf(x[15]));
#pragma unroll
  for (int off = kRowLanes / 2; off >= 1; off >>= 1)
    peak = max_nan(peak, __shfl_xor_sync(gmask, peak, off, kRowLanes));
  nonfinite |= !(peak <= 3.40282347e38f);  // a NaN or an infinity anywhere in the row
  const float s = peak > 0.f ? row_scale<FMT>(peak) : 1.0f;
  const float r = __frcp_rn(s);
  const bool fast_row = s >= 0x1p-90f;
  const uint32_t* w = reinterpret_cast<const uint32_t*>(raw);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t c[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int i = half * 8 + q * 4;
      float2 ya = make_float2(x[i], x[i + 1]);
      float2 yb = make_float2(x[i + 2], x[i + 3]);
      if (fast_row) {
        ya = div_rn_by2(ya, s, r);
        yb = div_rn_by2(yb, s, r);
      } else {
        ya = make_float2(__fdiv_rn(ya.x, s), __fdiv_rn(ya.y, s));
        yb = make_float2(__fdiv_rn(yb.x, s), __fdiv_rn(yb.y, s));
      }
      c[q] = codes4<FMT>(ya, yb, w[i / 2], w[i / 2 + 1]);
    }
    codes[half] = make_uint2(c[0], c[1]);
  }
  return s;
}

// One 8-lane group per (token, head) row of one batch entry (blockIdx.y), the K and V rows of
// a token together, ROWS rows per iteration (4 ROWS 16-byte loads in flight per lane before any
// arithmetic).  Row r = t * H + h; the group's (t, h) advance by the grid stride without a
// division.  Row indices are 32-bit (the launcher checks (L + L2) * H * 8 < 2^31).

__device__ __forceinline__ const __nv_bfloat16* append_src(const AppendParams& p, int which, int b, int t, int h,
                                                           int sub) {
  return t < p.L ? p.src[which] + b * p.s_b[which] + t * p.s_t[which] + h * p.s_h[which] + sub * 8
                 : p.src2[which] + b * p.s2_b[which] + (t - p.L) * p.s2_t[which] + h * p.s2_h[which] + sub * 8;
}

__device__ __forceinline__ void advance_row(int& t, int& h, int dt, int dh, int H) {
  t += dt;
  h += dh;
  if (h >= H) {
    h -= H;
    ++t;
  }
}

// ROWS rows per iteration: the loads of all of them (4 ROWS 16-byte loads per lane) are issued
// before any arithmetic.  ROWS = 1 (the default) keeps 64 registers and four blocks of 256
// threads per SM; ROWS = 2 holds twice the loads per lane at two blocks per SM (measured
// slower on the config-2 chunk: 32.7 against 28.2 us, as was a software prefetch of the next row).
template <int FMT, int ROWS>
__global__ void __launch_bounds__(256, ROWS == 1 ? 4 : 2) kv_append_kernel(const AppendParams p) {
  const int Lt = p.L + p.L2;
  const int b = blockIdx.y;
  const int sub = threadIdx.x & (kRowLanes - 1);
  // The four 8-lane groups of a warp own different rows and may leave the loop on different
  // iterations, so each group shuffles under its own lane mask.
  const unsigned gmask = 0xFFu << (threadIdx.x & 24);
  const int group = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) / kRowLanes);
  int t = group / p.H;
  int h = group - t * p.H;
  bool nonfinite = false;
  while (t < Lt) {
    int tt[ROWS], hh[ROWS];
    bool live[ROWS];
    uint4 raw[ROWS][2][2];
#pragma unroll
    for (int u = 0; u < ROWS; ++u) {
      tt[u] = t;
      hh[u] = h;
      live[u] = t < Lt;
      const int tl = live[u] ? t : 0;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint4* src = reinterpret_cast<const uint4*>(append_src(p, which, b, tl, h, 0));
        raw[u][which][0] = __ldg(src + sub);
        raw[u][which][1] = __ldg(src + 8 + sub);
      }
      advance_row(t, h, p.step_t, p.step_h, p.H);
    }
#pragma unroll
    for (int u = 0; u < ROWS; ++u) {
      if (!live[u]) continue;  // uniform over the 8-lane group that owns the row
      const long long dst_off = b * p.d_b + (tt[u] + p.start) * p.d_t + hh[u] * p.d_h + sub * 8;
      const long long sc_off = b * p.c_b + (tt[u] + p.start) * p.c_t + hh[u] * p.c_h;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        uint2 codes[2];
        const float s = quantise_row16<FMT>(raw[u][which], gmask, codes, nonfinite);
        uint8_t* dst = static_cast<uint8_t*>(p.dst[which]) + dst_off;
        *reinterpret_cast<uint2*>(dst) = codes[0];
        *reinterpret_cast<uint2*>(dst + 64) = codes[1];
        if (sub == 0) p.scale[which][sc_off] = s;
      }
    }
  }
  if (p.status != nullptr && __any_sync(0xffffffffu, nonfinite) && (threadIdx.x & 31) == 0)
    atomicOr(p.status, HYB_DEV_NONFINITE);
}

struct FiniteParams {
  const __nv_bfloat16* src;
  long long s_b, s_t, s_h;
  int B, L, H;
  int* status;
};

__global__ void __launch_bounds__(256) check_finite_kernel(const FiniteParams p) {
  const long long chunks = static_cast<long long>(p.B) * p.L * p.H * 16;
  bool bad = false;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int sub = static_cast<int>(c & 15);
    const long long row = c >> 4;
    const int h = static_cast<int>(row % p.H);
    const long long bt = row / p.H;
    const int t = static_cast<int>(bt % p.L);
    const int b = static_cast<int>(bt / p.L);
    uint4 raw = *reinterpret_cast<const uint4*>(p.src + b * p.s_b + t * p.s_t + h * p.s_h + sub * 8);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // bf16 exponent field all ones <=> inf or nan
      bad |= ((w[i] & 0x7F80u) == 0x7F80u) || ((w[i] & 0x7F800000u) == 0x7F800000u);
    }
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(p.status, HYB_DEV_NONFINITE);
}

struct DequantParams {
  int fmt;
  const void* src;
  long long s_b, s_t, s_h;
  const float* scale;
  long long c_b, c_t, c_h;
  int B, L, H;
  __nv_bfloat16* dst;  // contiguous [B, L, H, 128]
};

// bf16(code * scale) with one fp32 multiply and one RNE rounding, as in dequantize_kv's
// CPU branch (int8_kv_cache.py:202-204).
__global__ void __launch_bounds__(256) kv_dequant_kernel(const DequantParams p) {
  const long long chunks = static_cast<long long>(p.B) * p.L * p.H * 16;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int sub = static_cast<int>(c & 15);
    const long long row = c >> 4;
    const int h = static_cast<int>(row % p.H);
    const long long bt = row / p.H;
    const int t = static_cast<int>(bt % p.L);
    const int b = static_cast<int>(bt / p.L);
    const float s = p.scale[b * p.c_b + t * p.c_t + h * p.c_h];
    const uint8_t* src = static_cast<const uint8_t*>(p.src) + b * p.s_b + t * p.s_t + h * p.s_h + sub * 8;
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const uint8_t* bytes = reinterpret_cast<const uint8_t*>(&raw);
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a, bb;
      if (p.fmt == HYB_FMT_INT8) {
        a = static_cast<float>(static_cast<int8_t>(bytes[2 * i]));
        bb = static_cast<float>(static_cast<int8_t>(bytes[2 * i + 1]));
      } else {
        const __nv_fp8x2_storage_t pair =
            static_cast<__nv_fp8x2_storage_t>(bytes[2 * i] | (bytes[2 * i + 1] << 8));
        const __half2 hh = __half2(__nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3));
        const float2 f = __half22float2(hh);
        a = f.x;
        bb = f.y;
      }
      out[i] = pack_bf16x2(__fmul_rn(a, s), __fmul_rn(bb, s));
    }
    *reinterpret_cast<uint4*>(p.dst + row * 128 + sub * 8) = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

int grid_for(long long work_items, int threads) {
  long long blocks = (work_items + threads - 1) / threads;
  const long long cap = 148LL * 16;  // plenty of resident warps on 148 SMs
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace hyb

using namespace hyb;

extern "C" int hyb_kv_append_pair(int32_t fmt, int32_t B, int32_t L, int32_t H, int32_t D,
                                  int64_t cap, int64_t start, const hyb_tensor4* src_k,
                                  const hyb_tensor4* src_v, int32_t L2, const hyb_tensor4* src_k2,
                                  const hyb_tensor4* src_v2, void* dst_k, void* dst_v,
                                  int64_t d_sb, int64_t d_st, int64_t d_sh, float* scale_k,
                                  float* scale_v, int64_t s_sb, int64_t s_st, int64_t s_sh,
                                  int32_t* dev_status, void* stream) {
  if (fmt != HYB_FMT_E4M3 && fmt != HYB_FMT_INT8)
    return fail(HYB_ERR_UNSUPPORTED, "kv append: format %d is not E4M3 or INT8", fmt);
  if (D != 128) return fail(HYB_ERR_UNSUPPORTED, "kv append: head_dim %d != 128", D);
  if (B < 0 || L < 0 || L2 < 0 || H <= 0 || src_k == nullptr || src_v == nullptr ||
      (L2 > 0 && (src_k2 == nullptr || src_v2 == nullptr)))
    return fail(HYB_ERR_INVALID_ARG, "kv append: bad sizes or null views");
  if (start < 0 || start + L + L2 > cap)
    return fail(HYB_ERR_CAPACITY, "kv append: tokens [%lld, %lld) exceed capacity %lld",
                (long long)start, (long long)(start + L + L2), (long long)cap);
  if (L + L2 == 0 || B == 0) return HYB_OK;
  const hyb_tensor4* srcs[4] = {src_k, src_v, src_k2, src_v2};
  for (int i = 0; i < (L2 > 0 ? 4 : 2); ++i) {
    if (i < 2 && L == 0) continue;
    if (srcs[i]->fmt != HYB_FMT_BF16)
      return fail(HYB_ERR_INVALID_ARG, "kv append: sources must be bf16");
    if (!aligned16(srcs[i]->data) || (srcs[i]->s_b % 8) || (srcs[i]->s_t % 8) || (srcs[i]->s_h % 8))
      return fail(HYB_ERR_INVALID_ARG, "kv append: source rows must be 16-byte aligned");
  }
  if ((reinterpret_cast<uintptr_t>(dst_k) & 7u) || (reinterpret_cast<uintptr_t>(dst_v) & 7u) ||
      (d_sb % 8) || (d_st % 8) || (d_sh % 8))
    return fail(HYB_ERR_INVALID_ARG, "kv append: code rows must be 8-byte aligned");
  AppendParams p;
  p.fmt = fmt;
  p.L = L;
  p.L2 = L2;
  p.H = H;
  p.start = start;
  for (int i = 0; i < 2; ++i) {
    p.src[i] = static_cast<const __nv_bfloat16*>(srcs[i]->data);
    p.s_b[i] = srcs[i]->s_b;
    p.s_t[i] = srcs[i]->s_t;
    p.s_h[i] = srcs[i]->s_h;
    const hyb_tensor4* s2 = L2 > 0 ? srcs[2 + i] : srcs[i];
    p.src2[i] = static_cast<const __nv_bfloat16*>(s2->data);
    p.s2_b[i] = s2->s_b;
    p.s2_t[i] = s2->s_t;
    p.s2_h[i] = s2->s_h;
  }
  p.dst[0] = dst_k;
  p.dst[1] = dst_v;
  p.d_b = d_sb;
  p.d_t = d_st;
  p.d_h = d_sh;
  p.scale[0] = scale_k;
  p.scale[1] = scale_v;
  p.c_b = s_sb;
  p.c_t = s_st;
  p.c_h = s_sh;
  p.status = dev_status;
  const long long rows = static_cast<long long>(L + L2) * H;  // per batch entry
  if (rows * kRowLanes >= (1LL << 31) || B > 65535)
    return fail(HYB_ERR_UNSUPPORTED, "kv append: %lld rows x %d batch entries in one call (split the call)", rows,
                B);
  // about two iterations per group: enough loads in flight without a long grid-stride tail
  static const int rows_per_iter = [] {
    const char* e = getenv("HYB_APPEND_ROWS");
    return e != nullptr && atoi(e) == 2 ? 2 : 1;
  }();
  const long long per_block = 256 / kRowLanes;
  long long blocks = (rows + per_block * 2 * rows_per_iter - 1) / (per_block * 2 * rows_per_iter);
  blocks = blocks < 1 ? 1 : (blocks > 148LL * 64 ? 148LL * 64 : blocks);
  const long long stride = blocks * per_block;
  p.step_t = static_cast<int>(stride / H);
  p.step_h = static_cast<int>(stride % H);
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(B));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fmt == HYB_FMT_INT8) {
    if (rows_per_iter == 1)
      kv_append_kernel<HYB_FMT_INT8, 1><<<grid, 256, 0, st>>>(p);
    else
      kv_append_kernel<HYB_FMT_INT8, 2><<<grid, 256, 0, st>>>(p);
  } else {
    if (rows_per_iter == 1)
      kv_append_kernel<HYB_FMT_E4M3, 1><<<grid, 256, 0, st>>>(p);
    else
      kv_append_kernel<HYB_FMT_E4M3, 2><<<grid, 256, 0, st>>>(p);
  }
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_check_finite(const hyb_tensor4* src, int32_t B, int32_t L, int32_t H, int32_t D,
                                int32_t* dev_status, void* stream) {
  if (D != 128) return fail(HYB_ERR_UNSUPPORTED, "finite check: head_dim %d != 128", D);
  if (src == nullptr || dev_status == nullptr)
    return fail(HYB_ERR_INVALID_ARG, "finite check: null argument");
  if (src->fmt != HYB_FMT_BF16) return fail(HYB_ERR_INVALID_ARG, "finite check: bf16 only");
  if (!aligned16(src->data) || (src->s_b % 8) || (src->s_t % 8) || (src->s_h % 8))
    return fail(HYB_ERR_INVALID_ARG, "finite check: rows must be 16-byte aligned");
  if (B == 0 || L == 0) return HYB_OK;
  FiniteParams p{static_cast<const __nv_bfloat16*>(src->data), src->s_b, src->s_t, src->s_h, B, L, H,
                 dev_status};
  const long long chunks = static_cast<long long>(B) * L * H * 16;
  check_finite_kernel<<<grid_for(chunks, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_kv_dequant(const hyb_tensor4* src, int32_t B, int32_t valid, int32_t H,
                              int32_t D, void* dst, void* stream) {
  if (D != 128) return fail(HYB_ERR_UNSUPPORTED, "dequant: head_dim %d != 128", D);
  if (src == nullptr || dst == nullptr) return fail(HYB_ERR_INVALID_ARG, "dequant: null argument");
  if (src->fmt != HYB_FMT_E4M3 && src->fmt != HYB_FMT_INT8)
    return fail(HYB_ERR_UNSUPPORTED, "dequant: format %d is not E4M3 or INT8", src->fmt);
  if ((reinterpret_cast<uintptr_t>(src->data) & 7u) || (src->s_b % 8) || (src->s_t % 8) ||
      (src->s_h % 8) || !aligned16(dst))
    return fail(HYB_ERR_INVALID_ARG, "dequant: misaligned rows");
  if (B == 0 || valid == 0) return HYB_OK;
  DequantParams p{src->fmt, src->data, src->s_b, src->s_t, src->s_h, src->scale, src->ss_b,
                  src->ss_t, src->ss_h, B, valid, H, static_cast<__nv_bfloat16*>(dst)};
  const long long chunks = static_cast<long long>(B) * valid * H * 16;
  kv_dequant_kernel<<<grid_for(chunks, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}
