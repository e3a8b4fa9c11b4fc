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

constexpr int kRowLanes = 16;  // lanes per row: 16 x 8 bf16 = 128 values

struct AppendParams {
  int fmt;
  int B, L, L2, H;  // rows [0, L) from src, [L, L + L2) from src2
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
};

__device__ __forceinline__ void unpack8(const uint4& u, float (&x)[8]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(p[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// x / s rounded to nearest, from r = RN(1/s): q0 = RN(x r), then two residual steps
// q' = RN(q + r (x - s q)) with the residual formed exactly by the fma.  The first step
// leaves q1 within one ulp of x / s; correcting a quotient that close with a correctly
// rounded reciprocal gives RN(x / s) (P. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Develop. 34(1), 1990; restated in Muller
// et al., Handbook of Floating-Point Arithmetic, on FMA-based division).  The argument needs
// x, s and the residuals in the normal range: callers use it for |x|, s >= 2^-90 only.
__device__ __forceinline__ float div_rn_by(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float q1 = __fmaf_rn(__fmaf_rn(-s, q0, x), r, q0);
  return __fmaf_rn(__fmaf_rn(-s, q1, x), r, q1);
}

__device__ __forceinline__ float quotient(float x, float s, float r, bool fast_row) {
  if (fast_row && fabsf(x) >= 0x1p-90f) return div_rn_by(x, s, r);
  return __fdiv_rn(x, s);
}

// div_rn_by for a pair, in packed fp32x2 arithmetic (5 instructions for two quotients).  Valid
// for every x of a row whose scale s is at least 2^-90: the residuals x - s q stay normal unless
// |x| < 2^-103, and such an x has |x / s| < 2^-13, whose e4m3 and INT8 codes are 0 whatever
// the last bit of the quotient.
__device__ __forceinline__ float2 div_rn_by2(float2 x, float s, float r) {
  const float2 rr = make_float2(r, r);
  const float2 ns = make_float2(-s, -s);
  const float2 q0 = fmul2(x, rr);
  const float2 q1 = ffma2(ffma2(ns, q0, x), rr, q0);
  const float2 q2 = ffma2(ffma2(ns, q1, x), rr, q1);
  // A zero quotient takes the sign of x (-0 for a tiny negative x, as x / s gives): the last
  // step may add +0 to -0.  A nonzero quotient already has x's sign.
  return make_float2(__int_as_float(__float_as_int(q2.x) | (__float_as_int(x.x) & 0x80000000)),
                     __int_as_float(__float_as_int(q2.y) | (__float_as_int(x.y) & 0x80000000)));
}

// Quantise one 128-value row held by a 16-lane group (8 values per lane): absmax over the
// group, the row scale, and the 8 codes of this lane.  Returns the 8 code bytes.
__device__ __forceinline__ uint2 quantise_row8(const float (&x)[8], int fmt, unsigned half_mask, float& s_out,
                                               bool& nonfinite) {
  float peak = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    peak = fmaxf(peak, fabsf(x[i]));
    nonfinite |= !isfinite(x[i]);
  }
#pragma unroll
  for (int off = kRowLanes / 2; off >= 1; off >>= 1)
    peak = fmaxf(peak, __shfl_xor_sync(half_mask, peak, off, kRowLanes));
  const float denom = (fmt == HYB_FMT_INT8) ? 127.0f : 448.0f;
  const float s = peak > 0.f ? __fdiv_rn(peak, denom) : 1.0f;
  s_out = s;
  const bool fast_row = s >= 0x1p-90f;
  const float r = __frcp_rn(s);
  uint32_t w[2];
  if (fmt == HYB_FMT_INT8) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t acc = 0;
      float2 yp[2];
      if (fast_row) {
        yp[0] = div_rn_by2(make_float2(x[half * 4], x[half * 4 + 1]), s, r);
        yp[1] = div_rn_by2(make_float2(x[half * 4 + 2], x[half * 4 + 3]), s, r);
      } else {
        yp[0] = make_float2(__fdiv_rn(x[half * 4], s), __fdiv_rn(x[half * 4 + 1], s));
        yp[1] = make_float2(__fdiv_rn(x[half * 4 + 2], s), __fdiv_rn(x[half * 4 + 3], s));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float y = (i & 1) ? yp[i >> 1].y : yp[i >> 1].x;
        float r = (y >= 0.f) ? floorf(__fadd_rn(y, 0.5f)) : ceilf(__fsub_rn(y, 0.5f));
        r = fminf(fmaxf(r, -127.f), 127.f);
        const int8_t c = static_cast<int8_t>(static_cast<int>(r));
        acc |= static_cast<uint32_t>(static_cast<uint8_t>(c)) << (8 * i);
      }
      w[half] = acc;
    }
  } else {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t acc = 0;
#pragma unroll
      for (int i = 0; i < 4; i += 2) {
        // |x / s| <= 448 up to rounding, and the saturating conversion maps anything beyond to
        // +-448 exactly as a clamp would (a NaN row is flagged non-finite either way)
        const float2 xp = make_float2(x[half * 4 + i], x[half * 4 + i + 1]);
        const float2 y = fast_row ? div_rn_by2(xp, s, r) : make_float2(__fdiv_rn(xp.x, s), __fdiv_rn(xp.y, s));
        const __nv_fp8x2_storage_t c2 = __nv_cvt_float2_to_fp8x2(y, __NV_SATFINITE, __NV_E4M3);
        acc |= static_cast<uint32_t>(c2) << (8 * i);
      }
      w[half] = acc;
    }
  }
  return make_uint2(w[0], w[1]);
}

// One 16-lane group per (batch, token, head) row, K and V of the row together, two rows per
// iteration: four 16-byte loads in flight per lane before any arithmetic.  Row indices are
// 32-bit (the launcher checks B * (L + L2) * H * 16 < 2^31).
constexpr int kAppendRowsPerIter = 2;

__device__ __forceinline__ const __nv_bfloat16* append_src(const AppendParams& p, int which, int b, int t, int h,
                                                           int sub) {
  return t < p.L ? p.src[which] + b * p.s_b[which] + t * p.s_t[which] + h * p.s_h[which] + sub * 8
                 : p.src2[which] + b * p.s2_b[which] + (t - p.L) * p.s2_t[which] + h * p.s2_h[which] + sub * 8;
}

__global__ void __launch_bounds__(256) kv_append_kernel(const AppendParams p) {
  const int Lt = p.L + p.L2;
  const int rows = p.B * Lt * p.H;
  const int sub = threadIdx.x & (kRowLanes - 1);
  // The two 16-lane halves of a warp own different rows and may leave the loop on different
  // iterations, so each half shuffles under its own lane mask.
  const unsigned half_mask = (threadIdx.x & 16) ? 0xFFFF0000u : 0x0000FFFFu;
  const int group = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) / kRowLanes);
  const int groups = static_cast<int>(gridDim.x * blockDim.x / kRowLanes);
  bool nonfinite = false;
  for (int base = group; base < rows; base += groups * kAppendRowsPerIter) {
    int bb[kAppendRowsPerIter], tt[kAppendRowsPerIter], hh[kAppendRowsPerIter];
    bool live[kAppendRowsPerIter];
    uint4 raw[kAppendRowsPerIter][2];
#pragma unroll
    for (int u = 0; u < kAppendRowsPerIter; ++u) {
      const int row = base + u * groups;
      live[u] = row < rows;
      const int rr = live[u] ? row : base;
      hh[u] = rr % p.H;
      const int bt = rr / p.H;
      tt[u] = bt % Lt;
      bb[u] = bt / Lt;
#pragma unroll
      for (int which = 0; which < 2; ++which)
        raw[u][which] = __ldg(reinterpret_cast<const uint4*>(append_src(p, which, bb[u], tt[u], hh[u], sub)));
    }
#pragma unroll
    for (int u = 0; u < kAppendRowsPerIter; ++u) {
      if (!live[u]) continue;   // uniform over the 16-lane group that owns the row
      const long long dst_off = bb[u] * p.d_b + (tt[u] + p.start) * p.d_t + hh[u] * p.d_h + sub * 8;
      const long long sc_off = bb[u] * p.c_b + (tt[u] + p.start) * p.c_t + hh[u] * p.c_h;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        float x[8];
        unpack8(raw[u][which], x);
        float s;
        const uint2 codes = quantise_row8(x, p.fmt, half_mask, s, nonfinite);
        *reinterpret_cast<uint2*>(static_cast<uint8_t*>(p.dst[which]) + dst_off) = codes;
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
  p.B = B;
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
  const long long rows = static_cast<long long>(B) * (L + L2) * H;
  if (rows * kRowLanes >= (1LL << 31))
    return fail(HYB_ERR_UNSUPPORTED, "kv append: %lld rows in one call (split the call)", rows);
  // about two iterations per group: enough loads in flight without a long grid-stride tail
  long long blocks = (rows * kRowLanes + 256LL * 2 * kAppendRowsPerIter - 1) / (256LL * 2 * kAppendRowsPerIter);
  blocks = blocks < 1 ? 1 : (blocks > 148LL * 64 ? 148LL * 64 : blocks);
  kv_append_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
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
