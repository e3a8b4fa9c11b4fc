// Sequence-parallel data movement around the NCCL collectives, and the ring LSE merge.
//
//  * Ulysses pack: q, k, v [B, Ls, H, D] -> all_to_all send buffer [P, Ls_max, 3B, H/P, D],
//    the layout all_to_all_qkv builds with cat + reshape + transpose + contiguous
//    (hymm/distributed/communications.py:270-280, :113-124) and pack_qkv
//    (reactor/hy_nomas_fusions.py:9-78), in one pass.  Padding rows are zero.
//  * Ulysses unpack of O: receive buffer [P, H/P, Ls, B, D] -> [B, Ls, H, D]
//    (communications.py:191-198 after the head->sequence all_to_all).
//  * LSE merge of partial attentions (dynamic_ring_attention.py:86-105):
//    lse = max + log1p(exp(min - max)); out = out_a*exp(lse_a - lse) + out_b*exp(lse_b - lse).
#include <cstring>

#include "hyb_common.cuh"

namespace hyb {
namespace {

struct PackParams {
  int P, B, nsrc, Ls, Ls_max, H, Hp;
  const __nv_bfloat16* src0;
  const __nv_bfloat16* src1;
  const __nv_bfloat16* src2;
  long long s_b[3], s_t[3], s_h[3];
  __nv_bfloat16* send;
};

// One thread per 16-byte chunk of the send buffer [P, Ls_max, nsrc*B, H/P, D].
__global__ void __launch_bounds__(256) pack_qkv_kernel(const PackParams p) {
  const int nb = p.nsrc * p.B;
  const long long chunks = static_cast<long long>(p.P) * p.Ls_max * nb * p.Hp * 16;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int sub = static_cast<int>(c & 15);
    long long r = c >> 4;
    const int hl = static_cast<int>(r % p.Hp);
    r /= p.Hp;
    const int bb = static_cast<int>(r % nb);
    r /= nb;
    const int t = static_cast<int>(r % p.Ls_max);
    const int dst_rank = static_cast<int>(r / p.Ls_max);
    const int which = bb / p.B;
    const int b = bb % p.B;
    const int h = dst_rank * p.Hp + hl;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < p.Ls) {
      const __nv_bfloat16* src = which == 0 ? p.src0 : (which == 1 ? p.src1 : p.src2);
      const long long sb = which == 0 ? p.s_b[0] : (which == 1 ? p.s_b[1] : p.s_b[2]);
      const long long st = which == 0 ? p.s_t[0] : (which == 1 ? p.s_t[1] : p.s_t[2]);
      const long long sh = which == 0 ? p.s_h[0] : (which == 1 ? p.s_h[1] : p.s_h[2]);
      v = *reinterpret_cast<const uint4*>(src + b * sb + t * st + h * sh + sub * 8);
    }
    *reinterpret_cast<uint4*>(p.send + (c >> 4) * 128 + sub * 8) = v;
  }
}

constexpr int kMaxRanks = 64;

struct PackOParams {
  int P, B, Ls_max, Hp;
  int lens[kMaxRanks];
  int offs[kMaxRanks];
  const __nv_bfloat16* src;  // [B, L, Hp, D] strided
  long long s_b, s_t, s_h;
  __nv_bfloat16* send;       // [P, Hp, Ls_max, B, D]
};

__global__ void __launch_bounds__(256) pack_o_kernel(const PackOParams p) {
  const long long chunks = static_cast<long long>(p.P) * p.Hp * p.Ls_max * p.B * 16;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int sub = static_cast<int>(c & 15);
    long long r = c >> 4;
    const int b = static_cast<int>(r % p.B);
    r /= p.B;
    const int s = static_cast<int>(r % p.Ls_max);
    r /= p.Ls_max;
    const int hl = static_cast<int>(r % p.Hp);
    const int dst_rank = static_cast<int>(r / p.Hp);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (s < p.lens[dst_rank]) {
      const long long t = p.offs[dst_rank] + s;
      v = *reinterpret_cast<const uint4*>(p.src + b * p.s_b + t * p.s_t + hl * p.s_h + sub * 8);
    }
    *reinterpret_cast<uint4*>(p.send + (c >> 4) * 128 + sub * 8) = v;
  }
}

struct UnpackParams {
  int P, B, Ls, Ls_max, H, Hp;
  const __nv_bfloat16* recv;  // [P, Hp, Ls_max, B, D]
  __nv_bfloat16* out;
  long long o_b, o_t, o_h;
};

__global__ void __launch_bounds__(256) unpack_o_kernel(const UnpackParams p) {
  const long long chunks = static_cast<long long>(p.B) * p.Ls * p.H * 16;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int sub = static_cast<int>(c & 15);
    long long r = c >> 4;
    const int h = static_cast<int>(r % p.H);
    r /= p.H;
    const int t = static_cast<int>(r % p.Ls);
    const int b = static_cast<int>(r / p.Ls);
    const int src_rank = h / p.Hp;
    const int hl = h % p.Hp;
    const long long src_row = ((static_cast<long long>(src_rank) * p.Hp + hl) * p.Ls_max + t) * p.B + b;
    const uint4 v = *reinterpret_cast<const uint4*>(p.recv + src_row * 128 + sub * 8);
    *reinterpret_cast<uint4*>(p.out + b * p.o_b + t * p.o_t + h * p.o_h + sub * 8) = v;
  }
}

struct MergeParams {
  int rows, H, D;
  float* out_acc;        // [rows, H, D] fp32
  float* lse_acc;        // [H, rows] fp32
  const void* out_b;     // [rows, H, D] bf16 or fp32
  int out_b_fmt;         // 0 = bf16, 1 = fp32
  const float* lse_b;    // [H, rows]
};

// One warp per (row, head): D = 128 values, 4 per lane.
__global__ void __launch_bounds__(256) lse_merge_kernel(const MergeParams p) {
  const long long pairs = static_cast<long long>(p.rows) * p.H;
  const int lane = threadIdx.x & 31;
  for (long long i = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5; i < pairs;
       i += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const int h = static_cast<int>(i % p.H);
    const int row = static_cast<int>(i / p.H);
    const long long li = static_cast<long long>(h) * p.rows + row;
    const float la = p.lse_acc[li];
    const float lb = p.lse_b[li];
    const float mx = fmaxf(la, lb);
    const float mn = fminf(la, lb);
    float lse, wa, wb;
    if (mx == -INFINITY) {
      lse = -INFINITY;
      wa = 0.f;
      wb = 0.f;
    } else {
      lse = mx + log1pf(expf(mn - mx));
      wa = expf(la - lse);
      wb = expf(lb - lse);
    }
    float* oa = p.out_acc + i * p.D;
    for (int d = lane * 4; d < p.D; d += 128) {
      float4 a = *reinterpret_cast<float4*>(oa + d);
      float bv[4];
      if (p.out_b_fmt == 0) {
        const __nv_bfloat16* ob = static_cast<const __nv_bfloat16*>(p.out_b) + i * p.D + d;
        const uint2 raw = *reinterpret_cast<const uint2*>(ob);
        const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
        const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
        bv[0] = f0.x; bv[1] = f0.y; bv[2] = f1.x; bv[3] = f1.y;
      } else {
        const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(p.out_b) + i * p.D + d);
        bv[0] = f.x; bv[1] = f.y; bv[2] = f.z; bv[3] = f.w;
      }
      a.x = a.x * wa + bv[0] * wb;
      a.y = a.y * wa + bv[1] * wb;
      a.z = a.z * wa + bv[2] * wb;
      a.w = a.w * wa + bv[3] * wb;
      *reinterpret_cast<float4*>(oa + d) = a;
    }
    __syncwarp();
    if (lane == 0) p.lse_acc[li] = lse;
  }
}

int grid_for(long long items, int threads) {
  long long blocks = (items + threads - 1) / threads;
  const long long cap = 148LL * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }


// ---------------------------------------------------------------------------------------
// Peer-memory exchange (one process per GPU, buffers mapped into every rank with CUDA IPC).
//
// A push kernel writes this rank's slices straight into the destination ranks' buffers over
// NVLink, then the grid meets the other ranks at a flag barrier: every block fences its
// writes at system scope and counts itself in; the last block stores the next epoch into
// slot `rank` of every rank's flag array (release, system scope) and waits until every rank
// has stored that epoch into its own array (acquire loads, bounded: after kSpinLimitCycles
// it reports HYB_DEV_TIMEOUT in the status word and returns).  Epochs live in device memory,
// so a captured CUDA graph replays correctly.  Each rank visits its destinations starting
// from its own successor, so at any moment the ranks write to different peers.
// ---------------------------------------------------------------------------------------
struct PeerSync {
  int P, rank;
  int* flags[kMaxRanks];   // every rank's flag array int32[P], as mapped in this process
  unsigned* state;         // this rank: [0] blocks arrived in the current launch, [1] epoch
  int* status;
};

__device__ __forceinline__ void st_release_sys(int* ptr, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* ptr) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

__device__ void grid_signal_and_wait(const PeerSync& s) {
  __shared__ int is_last;
  __shared__ int epoch;
  __threadfence_system();  // every thread's peer writes, before the block counts itself in
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&s.state[0], 1u);
    is_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  if (threadIdx.x == 0) {
    __threadfence_system();
    s.state[0] = 0u;  // the next launch on this stream counts from zero
    s.state[1] += 1u;
    epoch = static_cast<int>(s.state[1]);
  }
  __syncthreads();
  const int e = epoch;
  const int t = threadIdx.x;
  if (t < s.P) {
    st_release_sys(s.flags[t] + s.rank, e);
    const int* mine = s.flags[s.rank] + t;
    const long long t0 = clock64();
    while (ld_acquire_sys(mine) < e) {
      if (clock64() - t0 > kSpinLimitCycles) {
        if (s.status != nullptr) atomicOr(s.status, HYB_DEV_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

struct PushQkvParams {
  int P, rank, B, Ls, Hp;
  const __nv_bfloat16* src[3];
  long long s_b[3], s_t[3], s_h[3];
  __nv_bfloat16* recv[kMaxRanks];  // each rank's receive buffer [P(src), Ls, 3B, H/P, D]
  PeerSync sync;
};

// One thread per 16-byte chunk: head slice of destination d of token t of q, k or v.
__global__ void __launch_bounds__(256) push_qkv_kernel(const PushQkvParams p) {
  const int nb = 3 * p.B;
  const long long per_dst = static_cast<long long>(p.Ls) * nb * p.Hp * 16;
  const long long chunks = per_dst * p.P;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(c / per_dst);
    long long r = c - k * per_dst;
    const int sub = static_cast<int>(r & 15);
    r >>= 4;
    const int hl = static_cast<int>(r % p.Hp);
    r /= p.Hp;
    const int bb = static_cast<int>(r % nb);
    const int t = static_cast<int>(r / nb);
    const int d = (p.rank + 1 + k) % p.P;
    const int which = bb / p.B;
    const int b = bb - which * p.B;
    const int h = d * p.Hp + hl;
    const uint4 v = *reinterpret_cast<const uint4*>(p.src[which] + b * p.s_b[which] + t * p.s_t[which] +
                                                    h * p.s_h[which] + sub * 8);
    __nv_bfloat16* dst = p.recv[d] + ((((static_cast<long long>(p.rank) * p.Ls + t) * nb + bb) * p.Hp + hl) * 128 + sub * 8);
    *reinterpret_cast<uint4*>(dst) = v;
  }
  grid_signal_and_wait(p.sync);
}

struct PushOParams {
  int P, rank, B, Ls, Lt, Hp, H;
  const __nv_bfloat16* o_send;  // this rank's heads, [P(dst), Hp, Ls, B, D]
  const __nv_bfloat16* txt;     // this rank's heads of the text rows [B, Lt, Hp, D] (strided)
  long long t_b, t_t, t_h;
  __nv_bfloat16* out[kMaxRanks];      // each rank's image output [B, Ls, H, D]
  __nv_bfloat16* txt_out[kMaxRanks];  // each rank's text output [B, Lt, H, D]
  PeerSync sync;
};

__global__ void __launch_bounds__(256) push_o_kernel(const PushOParams p) {
  const long long img_per_dst = static_cast<long long>(p.Hp) * p.Ls * p.B * 16;
  const long long txt_per_dst = static_cast<long long>(p.B) * p.Lt * p.Hp * 16;
  const long long chunks = (img_per_dst + txt_per_dst) * p.P;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < chunks;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    if (c < img_per_dst * p.P) {
      const int k = static_cast<int>(c / img_per_dst);
      long long r = c - k * img_per_dst;
      const int sub = static_cast<int>(r & 15);
      r >>= 4;
      const int b = static_cast<int>(r % p.B);
      r /= p.B;
      const int t = static_cast<int>(r % p.Ls);
      const int hl = static_cast<int>(r / p.Ls);
      const int d = (p.rank + 1 + k) % p.P;
      const uint4 v = *reinterpret_cast<const uint4*>(
          p.o_send + ((((static_cast<long long>(d) * p.Hp + hl) * p.Ls + t) * p.B + b) * 128 + sub * 8));
      *reinterpret_cast<uint4*>(p.out[d] + (((static_cast<long long>(b) * p.Ls + t) * p.H + p.rank * p.Hp + hl) * 128 +
                                            sub * 8)) = v;
    } else {
      const long long cc = c - img_per_dst * p.P;
      const int k = static_cast<int>(cc / txt_per_dst);
      long long r = cc - k * txt_per_dst;
      const int sub = static_cast<int>(r & 15);
      r >>= 4;
      const int hl = static_cast<int>(r % p.Hp);
      r /= p.Hp;
      const int t = static_cast<int>(r % p.Lt);
      const int b = static_cast<int>(r / p.Lt);
      const int d = (p.rank + 1 + k) % p.P;
      const uint4 v = *reinterpret_cast<const uint4*>(p.txt + b * p.t_b + t * p.t_t + hl * p.t_h + sub * 8);
      *reinterpret_cast<uint4*>(p.txt_out[d] + (((static_cast<long long>(b) * p.Lt + t) * p.H + p.rank * p.Hp + hl) * 128 +
                                                sub * 8)) = v;
    }
  }
  grid_signal_and_wait(p.sync);
}

struct PushBytesParams {
  int P, rank;
  long long chunks16;           // 16-byte chunks per destination
  const uint4* src;
  uint4* dst[kMaxRanks];        // where this rank's bytes go in each rank's buffer
  PeerSync sync;
};

// The same bytes to every rank (an all-gather contribution); destinations whose pointer is the
// source itself are skipped.
// Eight 16-byte chunks per thread and iteration, all loaded before any store, so that a grid
// of a few blocks (the overlapped ring schedule leaves the other SMs to an attention launch)
// still keeps enough bytes in flight to fill the links.
constexpr int kPushUnroll = 8;
__global__ void __launch_bounds__(256) push_bytes_kernel(const PushBytesParams p) {
  const long long total = p.chunks16 * p.P;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long c0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c0 < total;
       c0 += stride * kPushUnroll) {
    uint4 v[kPushUnroll];
#pragma unroll
    for (int u = 0; u < kPushUnroll; ++u) {
      const long long c = c0 + u * stride;
      if (c < total) {
        const int k = static_cast<int>(c / p.chunks16);
        v[u] = p.src[c - k * p.chunks16];
      }
    }
#pragma unroll
    for (int u = 0; u < kPushUnroll; ++u) {
      const long long c = c0 + u * stride;
      if (c < total) {
        const int k = static_cast<int>(c / p.chunks16);
        const int d = (p.rank + 1 + k) % p.P;
        if (p.dst[d] != p.src) p.dst[d][c - k * p.chunks16] = v[u];
      }
    }
  }
  grid_signal_and_wait(p.sync);
}

// A barrier alone (one block): every rank arrives when its stream reaches this launch, i.e.
// after every earlier kernel on it, and waits (bounded) for all the others.  Placed before a
// push into buffers that the other ranks read after the previous push's barrier, it orders
// their reads of the previous call before this call's writes.
__global__ void __launch_bounds__(64) barrier_kernel(const PeerSync s) { grid_signal_and_wait(s); }

int peer_sync_of(const hyb_peer_sync* ps, int P, int rank, PeerSync* out) {
  if (ps == nullptr || ps->state == nullptr) return fail(HYB_ERR_INVALID_ARG, "peer sync: null state");
  out->P = P;
  out->rank = rank;
  for (int r = 0; r < P; ++r) {
    if (ps->flags[r] == nullptr || (reinterpret_cast<uintptr_t>(ps->flags[r]) & 3u))
      return fail(HYB_ERR_INVALID_ARG, "peer sync: flag array of rank %d missing or misaligned", r);
    out->flags[r] = ps->flags[r];
  }
  out->state = ps->state;
  out->status = ps->dev_status;
  return HYB_OK;
}

}  // namespace
}  // namespace hyb

using namespace hyb;

extern "C" int hyb_ulysses_pack_qkv(int32_t P, int32_t B, int32_t Ls, int32_t Ls_max, int32_t H, int32_t D,
                                    const hyb_tensor4* q, const hyb_tensor4* k, const hyb_tensor4* v,
                                    void* send, void* stream) {
  if (D != 128) return fail(HYB_ERR_UNSUPPORTED, "ulysses pack: head_dim %d != 128", D);
  if (P <= 0 || B <= 0 || Ls < 0 || Ls_max < Ls || H <= 0 || H % P != 0)
    return fail(HYB_ERR_INVALID_ARG, "SP ranks require identical head counts divisible by SP size");
  if ((k == nullptr) != (v == nullptr)) return fail(HYB_ERR_INVALID_ARG, "ulysses pack: k and v go together");
  const int nsrc = k == nullptr ? 1 : 3;
  const hyb_tensor4* srcs[3] = {q, k, v};
  for (int i = 0; i < nsrc; ++i) {
    if (srcs[i] == nullptr || srcs[i]->fmt != HYB_FMT_BF16 || (Ls > 0 && !al16(srcs[i]->data)) ||
        (srcs[i]->s_b % 8) || (srcs[i]->s_t % 8) || (srcs[i]->s_h % 8))
      return fail(HYB_ERR_INVALID_ARG, "ulysses pack: bf16 16-byte aligned inputs required");
  }
  if (!al16(send)) return fail(HYB_ERR_INVALID_ARG, "ulysses pack: send buffer misaligned");
  if (Ls_max == 0) return HYB_OK;
  PackParams p;
  p.P = P;
  p.B = B;
  p.nsrc = nsrc;
  p.Ls = Ls;
  p.Ls_max = Ls_max;
  p.H = H;
  p.Hp = H / P;
  p.src0 = static_cast<const __nv_bfloat16*>(q->data);
  p.src1 = nsrc == 3 ? static_cast<const __nv_bfloat16*>(k->data) : nullptr;
  p.src2 = nsrc == 3 ? static_cast<const __nv_bfloat16*>(v->data) : nullptr;
  for (int i = 0; i < 3; ++i) {
    const hyb_tensor4* s = srcs[i < nsrc ? i : 0];
    p.s_b[i] = s->s_b;
    p.s_t[i] = s->s_t;
    p.s_h[i] = s->s_h;
  }
  p.send = static_cast<__nv_bfloat16*>(send);
  const long long chunks = static_cast<long long>(P) * Ls_max * nsrc * B * p.Hp * 16;
  pack_qkv_kernel<<<grid_for(chunks, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_ulysses_pack_o(int32_t P, int32_t B, const int32_t* lens, int32_t Ls_max, int32_t Hp, int32_t D,
                                  const hyb_tensor4* x, void* send, void* stream) {
  if (D != 128) return fail(HYB_ERR_UNSUPPORTED, "ulysses pack o: head_dim %d != 128", D);
  if (P <= 0 || P > kMaxRanks || B <= 0 || Hp <= 0 || Ls_max < 0 || lens == nullptr || x == nullptr)
    return fail(HYB_ERR_INVALID_ARG, "ulysses pack o: bad sizes (at most %d ranks)", kMaxRanks);
  PackOParams p;
  p.P = P;
  p.B = B;
  p.Ls_max = Ls_max;
  p.Hp = Hp;
  int off = 0;
  for (int r = 0; r < P; ++r) {
    if (lens[r] < 0 || lens[r] > Ls_max) return fail(HYB_ERR_INVALID_ARG, "ulysses pack o: bad length");
    p.lens[r] = lens[r];
    p.offs[r] = off;
    off += lens[r];
  }
  if (x->fmt != HYB_FMT_BF16 || (off > 0 && !al16(x->data)) || (x->s_b % 8) || (x->s_t % 8) || (x->s_h % 8) ||
      !al16(send))
    return fail(HYB_ERR_INVALID_ARG, "ulysses pack o: bf16 16-byte aligned buffers required");
  if (Ls_max == 0) return HYB_OK;
  p.src = static_cast<const __nv_bfloat16*>(x->data);
  p.s_b = x->s_b;
  p.s_t = x->s_t;
  p.s_h = x->s_h;
  p.send = static_cast<__nv_bfloat16*>(send);
  const long long chunks = static_cast<long long>(P) * Hp * Ls_max * B * 16;
  pack_o_kernel<<<grid_for(chunks, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_ulysses_unpack_o(int32_t P, int32_t B, int32_t Ls, int32_t Ls_max, int32_t H, int32_t D,
                                    const void* recv, void* out, int64_t o_sb, int64_t o_st, int64_t o_sh,
                                    void* stream) {
  if (D != 128) return fail(HYB_ERR_UNSUPPORTED, "ulysses unpack: head_dim %d != 128", D);
  if (P <= 0 || B <= 0 || Ls < 0 || Ls_max < Ls || H <= 0 || H % P != 0)
    return fail(HYB_ERR_INVALID_ARG, "ulysses unpack: bad sizes");
  if (!al16(recv) || !al16(out) || (o_sb % 8) || (o_st % 8) || (o_sh % 8))
    return fail(HYB_ERR_INVALID_ARG, "ulysses unpack: misaligned buffers");
  if (Ls == 0) return HYB_OK;
  UnpackParams p{P, B, Ls, Ls_max, H, H / P, static_cast<const __nv_bfloat16*>(recv),
                 static_cast<__nv_bfloat16*>(out), o_sb, o_st, o_sh};
  const long long chunks = static_cast<long long>(B) * Ls * H * 16;
  unpack_o_kernel<<<grid_for(chunks, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_lse_merge(int32_t rows, int32_t H, int32_t D, float* out_acc, float* lse_acc,
                             const void* out_b, int32_t out_b_fmt, const float* lse_b, void* stream) {
  if (D != 128) return fail(HYB_ERR_UNSUPPORTED, "lse merge: head_dim %d != 128", D);
  if (rows < 0 || H <= 0 || out_acc == nullptr || lse_acc == nullptr || out_b == nullptr || lse_b == nullptr ||
      (out_b_fmt != 0 && out_b_fmt != 1))
    return fail(HYB_ERR_INVALID_ARG, "lse merge: bad arguments");
  if (!al16(out_acc) || !al16(out_b)) return fail(HYB_ERR_INVALID_ARG, "lse merge: misaligned outputs");
  if (rows == 0) return HYB_OK;
  MergeParams p{rows, H, D, out_acc, lse_acc, out_b, out_b_fmt, lse_b};
  const long long threads = static_cast<long long>(rows) * H * 32;
  lse_merge_kernel<<<grid_for(threads, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
  if (ptr == nullptr || ipc_handle == nullptr || bytes <= 0) return fail(HYB_ERR_INVALID_ARG, "peer alloc: bad arguments");
  *ptr = nullptr;
  HYB_CUDA_TRY(cudaMalloc(ptr, static_cast<size_t>(bytes)));
  HYB_CUDA_TRY(cudaMemset(*ptr, 0, static_cast<size_t>(bytes)));
  cudaIpcMemHandle_t h;
  HYB_CUDA_TRY(cudaIpcGetMemHandle(&h, *ptr));
  memcpy(ipc_handle, &h, sizeof(h));
  return HYB_OK;
}

extern "C" int hyb_peer_open(const void* ipc_handle, void** peer_ptr) {
  if (ipc_handle == nullptr || peer_ptr == nullptr) return fail(HYB_ERR_INVALID_ARG, "peer open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  *peer_ptr = nullptr;
  HYB_CUDA_TRY(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return HYB_OK;
}

extern "C" int hyb_peer_close(void* peer_ptr) {
  if (peer_ptr == nullptr) return HYB_OK;
  HYB_CUDA_TRY(cudaIpcCloseMemHandle(peer_ptr));
  return HYB_OK;
}

extern "C" int hyb_peer_free(void* ptr) {
  if (ptr == nullptr) return HYB_OK;
  HYB_CUDA_TRY(cudaFree(ptr));
  return HYB_OK;
}

extern "C" int hyb_ulysses_push_qkv(int32_t P, int32_t rank, int32_t B, int32_t Ls, int32_t H, int32_t D,
                                    const hyb_tensor4* q, const hyb_tensor4* k, const hyb_tensor4* v,
                                    void* const* recv, const hyb_peer_sync* sync, void* stream) {
  if (D != 128) return fail(HYB_ERR_UNSUPPORTED, "ulysses push: head_dim %d != 128", D);
  if (P <= 1 || P > kMaxRanks || rank < 0 || rank >= P || B <= 0 || Ls < 0 || H <= 0 || H % P != 0 ||
      q == nullptr || k == nullptr || v == nullptr || recv == nullptr)
    return fail(HYB_ERR_INVALID_ARG, "ulysses push: bad sizes (2..%d ranks, heads divisible by ranks)", kMaxRanks);
  PushQkvParams p;
  p.P = P;
  p.rank = rank;
  p.B = B;
  p.Ls = Ls;
  p.Hp = H / P;
  const hyb_tensor4* srcs[3] = {q, k, v};
  for (int i = 0; i < 3; ++i) {
    if (srcs[i]->fmt != HYB_FMT_BF16 || !al16(srcs[i]->data) || (srcs[i]->s_b % 8) || (srcs[i]->s_t % 8) ||
        (srcs[i]->s_h % 8))
      return fail(HYB_ERR_INVALID_ARG, "ulysses push: bf16 16-byte aligned q/k/v required");
    p.src[i] = static_cast<const __nv_bfloat16*>(srcs[i]->data);
    p.s_b[i] = srcs[i]->s_b;
    p.s_t[i] = srcs[i]->s_t;
    p.s_h[i] = srcs[i]->s_h;
  }
  for (int r = 0; r < P; ++r) {
    if (recv[r] == nullptr || !al16(recv[r])) return fail(HYB_ERR_INVALID_ARG, "ulysses push: receive buffer %d", r);
    p.recv[r] = static_cast<__nv_bfloat16*>(recv[r]);
  }
  int rc = peer_sync_of(sync, P, rank, &p.sync);
  if (rc != HYB_OK) return rc;
  const long long chunks = static_cast<long long>(P) * Ls * 3 * B * p.Hp * 16;
  push_qkv_kernel<<<grid_for(chunks > 0 ? chunks : 1, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_ulysses_push_o(int32_t P, int32_t rank, int32_t B, int32_t Ls, int32_t Lt, int32_t H, int32_t D,
                                  const void* o_send, const hyb_tensor4* txt, void* const* out, void* const* txt_out,
                                  const hyb_peer_sync* sync, void* stream) {
  if (D != 128) return fail(HYB_ERR_UNSUPPORTED, "ulysses push o: head_dim %d != 128", D);
  if (P <= 1 || P > kMaxRanks || rank < 0 || rank >= P || B <= 0 || Ls < 0 || Lt < 0 || H <= 0 || H % P != 0 ||
      out == nullptr || (Lt > 0 && (txt == nullptr || txt_out == nullptr)) || (Ls > 0 && !al16(o_send)))
    return fail(HYB_ERR_INVALID_ARG, "ulysses push o: bad sizes or buffers");
  PushOParams p;
  p.P = P;
  p.rank = rank;
  p.B = B;
  p.Ls = Ls;
  p.Lt = Lt;
  p.Hp = H / P;
  p.H = H;
  p.o_send = static_cast<const __nv_bfloat16*>(o_send);
  p.txt = nullptr;
  p.t_b = p.t_t = p.t_h = 0;
  if (Lt > 0) {
    if (txt->fmt != HYB_FMT_BF16 || !al16(txt->data) || (txt->s_b % 8) || (txt->s_t % 8) || (txt->s_h % 8))
      return fail(HYB_ERR_INVALID_ARG, "ulysses push o: bf16 16-byte aligned text rows required");
    p.txt = static_cast<const __nv_bfloat16*>(txt->data);
    p.t_b = txt->s_b;
    p.t_t = txt->s_t;
    p.t_h = txt->s_h;
  }
  for (int r = 0; r < P; ++r) {
    if (out[r] == nullptr || !al16(out[r]) || (Lt > 0 && (txt_out[r] == nullptr || !al16(txt_out[r]))))
      return fail(HYB_ERR_INVALID_ARG, "ulysses push o: output buffer %d", r);
    p.out[r] = static_cast<__nv_bfloat16*>(out[r]);
    p.txt_out[r] = Lt > 0 ? static_cast<__nv_bfloat16*>(txt_out[r]) : nullptr;
  }
  int rc = peer_sync_of(sync, P, rank, &p.sync);
  if (rc != HYB_OK) return rc;
  const long long chunks = static_cast<long long>(P) * (static_cast<long long>(p.Hp) * Ls * B + static_cast<long long>(B) * Lt * p.Hp) * 16;
  push_o_kernel<<<grid_for(chunks > 0 ? chunks : 1, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_peer_barrier(int32_t P, int32_t rank, const hyb_peer_sync* sync, void* stream) {
  if (P <= 1 || P > kMaxRanks || rank < 0 || rank >= P)
    return fail(HYB_ERR_INVALID_ARG, "peer barrier: bad arguments (2..%d ranks)", kMaxRanks);
  PeerSync s;
  int rc = peer_sync_of(sync, P, rank, &s);
  if (rc != HYB_OK) return rc;
  barrier_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(s);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_peer_push_bytes_n(int32_t P, int32_t rank, const void* src, int64_t bytes, void* const* dst,
                                     const hyb_peer_sync* sync, int32_t max_blocks, void* stream);

extern "C" int hyb_peer_push_bytes(int32_t P, int32_t rank, const void* src, int64_t bytes, void* const* dst,
                                   const hyb_peer_sync* sync, void* stream) {
  return hyb_peer_push_bytes_n(P, rank, src, bytes, dst, sync, 0, stream);
}

extern "C" int hyb_peer_push_bytes_n(int32_t P, int32_t rank, const void* src, int64_t bytes, void* const* dst,
                                     const hyb_peer_sync* sync, int32_t max_blocks, void* stream) {
  if (P <= 1 || P > kMaxRanks || rank < 0 || rank >= P || bytes < 0 || (bytes % 16) != 0 || dst == nullptr ||
      (bytes > 0 && !al16(src)))
    return fail(HYB_ERR_INVALID_ARG, "peer push: bad arguments (16-byte multiples, 2..%d ranks)", kMaxRanks);
  PushBytesParams p;
  p.P = P;
  p.rank = rank;
  p.chunks16 = bytes / 16;
  p.src = static_cast<const uint4*>(src);
  for (int r = 0; r < P; ++r) {
    if (dst[r] == nullptr || !al16(dst[r])) return fail(HYB_ERR_INVALID_ARG, "peer push: destination %d", r);
    p.dst[r] = static_cast<uint4*>(dst[r]);
  }
  int rc = peer_sync_of(sync, P, rank, &p.sync);
  if (rc != HYB_OK) return rc;
  const long long total = p.chunks16 * P;
  int blocks = grid_for(total > 0 ? total : 1, 256);
  if (max_blocks > 0 && blocks > max_blocks) blocks = max_blocks;
  push_bytes_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}
