// Chunk-causal cached attention for sm_100a.
//
//  * stage kernels: compose the key sequence [visible history | current image | current
//    text] head-major in bf16 (history decoded from E4M3 / INT8 codes with its per-token
//    per-head scale), the query sequence [image | text], and the key / query visibility
//    bitmaps.  This replaces dequantize_kv + torch.cat + unpad of
//    causal_attention_with_cache_mp (hymm/models/dit/nomas_cpt.py:520-531, :608-685,
//    :807-817) and the compact_kv gather of reactor/hy_nomas_cache.py:48-73.
//  * attention kernel: one CTA per (128-query tile, head, batch); a TMA producer warp,
//    a single-thread tcgen05 MMA issuer, and one softmax/epilogue warpgroup.
//    S = Q K^T and O += P V run on the tensor cores with fp32 accumulators in tensor
//    memory (S double-buffered, 2 x 128 columns; O 128 columns); K/V tiles stream
//    through a 2-stage shared-memory ring.  Online softmax with lazy rescaling (O is
//    only rescaled when the running max grows by more than 2^8), frame-level
//    block-causal masking with fully masked key tiles skipped, and key/query validity
//    bitmaps for padded history and text.  The output is written at its final
//    position (pad_tokens semantics: masked text queries produce zero rows).
#include <limits.h>

#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <queue>
#include <vector>

#include "hyb_common.cuh"

namespace hyb {
namespace {

constexpr int kBM = 128;                    // query rows per tile
constexpr int kBN = 128;                    // keys per tile
constexpr int kHD = 128;                    // head dim
constexpr int kStages = 2;                  // K/V shared-memory ring depth
constexpr int kTileBytes = kBM * kHD * 2;   // one 128 x 128 bf16 tile
constexpr int kHalfTile = kTileBytes / 2;   // one 64-column TMA box (128-byte rows)
constexpr uint32_t kTmemCols = 512;         // S0 [0,128) S1 [128,256) O [256,384)
constexpr uint32_t kTmemO = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;   // log2 units

struct AttnKParams {
  // Lq queries: Li image rows then text rows.  Lk keys: Lh history, Lik image, then text.
  int B, H, Lq, Lk, Lh, Li, Lik, gtok;
  // Global token positions for the block-causal rule: image query i sees image key j iff
  // kpos(j) / gtok <= qpos(i) / gtok.  Positions come in up to two increasing segments
  // (a zig-zag ring shard holds two chunks of the sequence): qpos(i) = q_pos0 + i for
  // i < q_seg, else q_pos1 + (i - q_seg); kpos likewise with k_seg / k_pos1.  A chunk
  // attending to itself has one segment at 0.
  int q_pos0, k_pos0, q_seg, q_pos1, k_seg, k_pos1;
  float scale_log2;
  const uint32_t* kbits;
  int kwords;
  const uint32_t* qbits;
  int qwords;
  __nv_bfloat16* out_img;
  long long oi_b, oi_t, oi_h, oi_seg, oi_sseg;
  __nv_bfloat16* out_txt;
  long long ot_b, ot_t, ot_h;
  float* lse;
  int* status;
  int num_qtiles;
  // Split-KV: a query pair split into k > 1 key slices writes, per slice, normalised fp32
  // partial rows part_o [S, B, H, Lq, 128] (S = kv_splits, the buffers' capacity, >= k) and
  // their natural-log LSE part_lse [S, B, H, Lq]; merge_splits_kernel combines them.
  int kv_splits;
  float* part_o;
  float* part_lse;
  // Ring accumulator (all queries image rows): acc_o fp32 [B, Lq, H, 128], acc_lse fp32
  // [B, H, Lq].  acc_mode bit 0: merge with its contents; bit 1: write the merged rows as
  // bf16 to out_img (+ lse) instead of back to the accumulator.
  float* acc_o;
  float* acc_lse;
  int acc_mode;
  // Partial rows scattered to their owner ranks (hyb_part_scatter), active when sc_o is set:
  // image row q to rank q / sc_rows, row q % sc_rows; text row t to every rank, row sc_rows + t;
  // partial index sc_index0 + this CTA's key slice.
  float* const* sc_o;
  float* const* sc_lse;
  int sc_ranks, sc_rows, sc_index0;
};

__host__ __device__ __forceinline__ int imin(int a, int b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int imax(int a, int b) { return a > b ? a : b; }

__host__ __device__ __forceinline__ long long q_position(const AttnKParams& p, int i) {
  return i < p.q_seg ? static_cast<long long>(p.q_pos0) + i : static_cast<long long>(p.q_pos1) + (i - p.q_seg);
}

// Image keys visible to an image query at global position qpos.  Key positions increase with
// the key index, so the visible image keys are the prefix [0, count).
__host__ __device__ __forceinline__ int img_keys_visible(const AttnKParams& p, long long qpos) {
  const long long lim = (qpos / p.gtok + 1) * p.gtok;  // first position of a later group
  long long a = lim - p.k_pos0;
  a = a < 0 ? 0 : (a > p.k_seg ? p.k_seg : a);
  const long long n1 = p.Lik - p.k_seg;
  long long c = lim - p.k_pos1;
  c = c < 0 ? 0 : (c > n1 ? n1 : c);
  return static_cast<int>(a + c);
}

// Log-sum-exp merge of a running ring output (LSE lse_a) with one step's normalised rows
// (LSE lse_b): merged = wa * acc + wb * step, LSE of the union.  Both weights are zero when
// neither side has seen a visible key.
struct AccWeights {
  float wa, wb, lse;
};
__device__ __forceinline__ AccWeights acc_weights(float lse_a, float lse_b) {
  AccWeights w;
  const float m = fmaxf(lse_a, lse_b);
  if (m == -INFINITY) {
    w.wa = 0.f;
    w.wb = 0.f;
    w.lse = -INFINITY;
    return w;
  }
  const float ea = __expf(lse_a - m);
  const float eb = __expf(lse_b - m);
  const float sum = ea + eb;
  const float inv = 1.f / sum;
  w.wa = ea * inv;
  w.wb = eb * inv;
  w.lse = m + __logf(sum);
  return w;
}

// Key tiles visited by one query tile: [0, a_end) then [b_begin, b_end).
// Image keys past the block-causal limit of the tile's last row are never loaded.
struct TileRange {
  int a_end, b_begin, b_end;
  __host__ __device__ int count() const { return a_end + (b_end - b_begin); }
  __host__ __device__ int tile(int j) const { return j < a_end ? j : b_begin + (j - a_end); }
};

__host__ __device__ TileRange key_tiles(const AttnKParams& p, int q0, int rows = kBM) {
  const int q_last = imin(q0 + rows, p.Lq) - 1;
  const int ntk = (p.Lk + kBN - 1) / kBN;
  int img_vis_end = p.Lh + p.Lik;
  if (p.gtok > 0 && q_last < p.Li) img_vis_end = p.Lh + img_keys_visible(p, q_position(p, q_last));
  TileRange r;
  r.a_end = imin((img_vis_end + kBN - 1) / kBN, ntk);
  const int txt_begin = p.Lh + p.Lik;
  if (txt_begin < p.Lk) {
    r.b_begin = imax(txt_begin / kBN, r.a_end);
    r.b_end = ntk;
  } else {
    r.b_begin = 0;
    r.b_end = 0;
  }
  return r;
}

// Work list of one launch.  CTA x runs unit x of the head-major list
//   for bh in [0, B*H):  for i in [0, npairs) (query pair npairs-1-i: heaviest first):
//     for k in [0, k_i):  key slice k of k_i of that pair
// so that a heavy pair is cut into more slices than a light one and every CTA gets about the
// same number of key tiles.  prefix[i] = k_0 + ... + k_{i-1}; per_bh = prefix[npairs].
// uniform > 0 stands for k_i = uniform for every pair (no table).
constexpr int kMaxPairTab = 512;
struct UnitMap {
  int npairs, per_bh, uniform, max_k;
  int prefix[kMaxPairTab + 1];
};

__device__ __forceinline__ int splits_of_pair(const UnitMap& um, int i) {
  return um.uniform > 0 ? um.uniform : um.prefix[i + 1] - um.prefix[i];
}

__device__ __forceinline__ void unit_of(const UnitMap& um, int x, int& bh, int& i, int& k, int& ki) {
  bh = x / um.per_bh;
  const int r = x - bh * um.per_bh;
  if (um.uniform > 0) {
    i = r / um.uniform;
    k = r - i * um.uniform;
    ki = um.uniform;
    return;
  }
  int lo = 0, hi = um.npairs - 1;  // largest i with prefix[i] <= r (prefix increases strictly)
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (um.prefix[mid] <= r) {
      lo = mid;
    } else {
      hi = mid - 1;
    }
  }
  i = lo;
  k = r - um.prefix[i];
  ki = um.prefix[i + 1] - um.prefix[i];
}

// Epilogue stores through a per-warp 4 KB shared-memory buffer.  A warp holds 32 rows (lane =
// row) of 32 columns; written directly, every store instruction would touch 32 rows with 16
// bytes each.  Transposed through shared memory (16-byte granules XOR-swizzled by row, no bank
// conflicts), each instruction writes whole 128-byte (fp32) or 64-byte (bf16) row chunks.
// fp32: row r of the warp goes to base + r * kHD (rows contiguous, as the split partials are);
// rows with r >= nrows are not written.
__device__ __forceinline__ void warp_store_f32_rows(uint8_t* ebuf, const float (&v)[32], float* base, int nrows,
                                                    int lane) {
#pragma unroll
  for (int g = 0; g < 8; ++g)
    *reinterpret_cast<float4*>(ebuf + lane * 128 + ((g ^ (lane & 7)) << 4)) =
        make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
  __syncwarp();
  const int g = lane & 7;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    const float4 x = *reinterpret_cast<const float4*>(ebuf + r * 128 + ((g ^ (r & 7)) << 4));
    if (r < nrows) reinterpret_cast<float4*>(base + static_cast<size_t>(r) * kHD)[g] = x;
  }
  __syncwarp();
}
// bf16: 16 packed pairs per lane; row r goes to the row pointer held by lane r (null: skip).
__device__ __forceinline__ void warp_store_bf16_rows(uint8_t* ebuf, const uint32_t (&o)[16], __nv_bfloat16* dst,
                                                     int lane) {
#pragma unroll
  for (int g = 0; g < 4; ++g)
    *reinterpret_cast<uint4*>(ebuf + lane * 64 + ((g ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(o[4 * g], o[4 * g + 1], o[4 * g + 2], o[4 * g + 3]);
  __syncwarp();
  const int g = lane & 3;
  const unsigned long long mine = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane >> 2);
    const uint4 x = *reinterpret_cast<const uint4*>(ebuf + r * 64 + ((g ^ ((r >> 1) & 3)) << 4));
    const unsigned long long d = __shfl_sync(0xffffffffu, mine, r);
    if (d != 0ull) reinterpret_cast<uint4*>(d)[g] = x;
  }
  __syncwarp();
}

// fp32 rows of 32 columns, row r to the row pointer held by lane r (null: skip).
__device__ __forceinline__ void warp_store_f32_rows_to(uint8_t* ebuf, const float (&v)[32], float* dst, int lane) {
#pragma unroll
  for (int g = 0; g < 8; ++g)
    *reinterpret_cast<float4*>(ebuf + lane * 128 + ((g ^ (lane & 7)) << 4)) =
        make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
  __syncwarp();
  const int g = lane & 7;
  const unsigned long long mine = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    const float4 x = *reinterpret_cast<const float4*>(ebuf + r * 128 + ((g ^ (r & 7)) << 4));
    const unsigned long long d = __shfl_sync(0xffffffffu, mine, r);
    if (d != 0ull) reinterpret_cast<float4*>(d)[g] = x;
  }
  __syncwarp();
}

// Bounded wait that ignores the abort flag (used to drain in-flight async work on exit).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kSpinLimitCycles) break;
  }
}

// ======================================================================================
// Two query tiles per CTA (256 rows of one head): the K/V tiles are loaded once for both,
// and the single MMA thread alternates between the two softmax warpgroups so the tensor
// pipe computes one tile's S = QK^T / O += PV while the other warpgroup exponentiates.
// Warpgroup 0: warp 0 TMA producer, warp 1 MMA issuer (warps 2-3 idle); warpgroups 1 and
// 2: softmax + epilogue of query tile 0 / 1 (a warp accesses the tensor-memory lane quarter
// warp % 4).  A whole 128-column row of S is held in registers within the 168-register
// budget of 384 threads (four max chains, O rescaled after P is written).
// Tensor memory: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512); P_i overwrites S_i.
// ======================================================================================
constexpr int kThreads2 = 384;  // warps 0-3: TMA / MMA / idle, warps 4-7 and 8-11 softmax
constexpr int kPairRows = 2 * kBM;
// The key-visibility bitmap of the CTA's batch row is staged in shared memory when it
// fits (keys <= 32 * kMaxSmemBitWords); otherwise the softmax reads it through L1.
constexpr int kMaxSmemBitWords = 4096;

// kEmuPer8: that many eighths of a row's 64 score pairs take exp2 on the FMA pipe
// (exp2_poly2) and the rest on MUFU, to balance the two units against the tensor pipe.  The
// emulated pairs are the last ones of the row, computed when most scores are already
// consumed, so the polynomial's temporaries do not raise register pressure.
// kVF16: V staged in fp16 and P rounded to fp16 for P.V (else both bf16).
template <int kEmuPer8, bool kVF16>
__global__ void __launch_bounds__(kThreads2, 1)
    attn_fwd2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnKParams p,
                     const __grid_constant__ UnitMap um) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                              // [2][kTileBytes]
  uint8_t* sK = sQ + 2 * kTileBytes;               // [kStages][kTileBytes]
  uint8_t* sV = sK + kStages * kTileBytes;         // [kStages][kTileBytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kStages * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;            // [kStages]: K and V of the tile landed
  uint64_t* kv_empty = kv_full + kStages;  // [kStages]: every MMA reading the stage completed
  uint64_t* s_full = kv_empty + kStages;   // [2] one per query tile
  uint64_t* p_full = s_full + 2;         // [2]
  uint64_t* o_full = p_full + 2;         // [1]
  uint64_t* mma_done = o_full + 1;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* sBits = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(bars) + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Head-major work list (CTAs resident together share one head's K/V in L2), heaviest
  // query pair of each head first.
  int bh, ipair, split, nsplit;
  unit_of(um, static_cast<int>(blockIdx.x), bh, ipair, split, nsplit);
  const int qp = um.npairs - 1 - ipair;
  const int h = bh % p.H;
  const int b = bh / p.H;
  const int q0 = qp * kPairRows;
  const bool has1 = q0 + kBM < p.Lq;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    mbar_init(o_full, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  const bool bits_in_smem = p.kwords <= kMaxSmemBitWords;
  const uint32_t* kb_glob = p.kbits + static_cast<size_t>(b) * p.kwords;
  if (bits_in_smem) {
    for (int i = threadIdx.x; i < p.kwords / 4; i += blockDim.x)
      reinterpret_cast<uint4*>(sBits)[i] = __ldg(reinterpret_cast<const uint4*>(kb_glob) + i);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const TileRange tr = key_tiles(p, q0, kPairRows);
  // This CTA's slice [j_begin, j_begin + n) of the pair's key-tile list.
  const int n_all = tr.count();
  const int j_begin = static_cast<int>((static_cast<long long>(n_all) * split) / nsplit);
  const int n = static_cast<int>((static_cast<long long>(n_all) * (split + 1)) / nsplit) - j_begin;

  if (warp < 4) {
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------- TMA producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_expect_tx(q_full, has1 ? 2 * kTileBytes : kTileBytes);
      tma_load_3d(sQ, &tmQ, q_full, 0, q0, bh);
      tma_load_3d(sQ + kHalfTile, &tmQ, q_full, 64, q0, bh);
      if (has1) {
        tma_load_3d(sQ + kTileBytes, &tmQ, q_full, 0, q0 + kBM, bh);
        tma_load_3d(sQ + kTileBytes + kHalfTile, &tmQ, q_full, 64, q0 + kBM, bh);
      }
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int k0 = tr.tile(j_begin + j) * kBN;
        const int st = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, abort_flag)) break;
        mbar_expect_tx(&kv_full[st], 2 * kTileBytes);
        tma_load_3d(sK + st * kTileBytes, &tmK, &kv_full[st], 0, k0, bh);
        tma_load_3d(sK + st * kTileBytes + kHalfTile, &tmK, &kv_full[st], 64, k0, bh);
        tma_load_3d(sV + st * kTileBytes, &tmV, &kv_full[st], 0, k0, bh);
        tma_load_3d(sV + st * kTileBytes + kHalfTile, &tmV, &kv_full[st], 64, k0, bh);
        issued = j + 1;
      }
      if (*abort_flag) {
        mbar_drain(q_full, 0);
        for (int j = max(0, issued - kStages); j < issued; ++j) mbar_drain(&kv_full[j % kStages], (j / kStages) & 1);
      }
    } else if (warp == 1 && lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      // The issuing thread shares its SM sub-partition with two softmax warps, and every
      // mbarrier operation costs it on the order of 100 cycles during which the tensor pipe
      // can drain, so it waits and commits as little as possible (one K/V wait and one
      // stage-free commit per key tile) and forms each operand descriptor as a base plus a
      // constant.
      constexpr uint32_t kIdescQK = idesc_bf16_f32(kBM, kBN, false, false);
      constexpr uint32_t kIdescPV =
          kVF16 ? idesc_f16_f32(kBM, kHD, false, true) : idesc_bf16_f32(kBM, kHD, false, true);
      const SDesc dq = sdesc_sw128_parts(smem_u32(sQ), 16, 1024);
      const SDesc dk = sdesc_sw128_parts(smem_u32(sK), 16, 1024);
      const SDesc dv = sdesc_sw128_parts(smem_u32(sV), kHalfTile, 1024);
      auto issue_qk = [&](int qi, int st) {
        const uint32_t d = tmem + static_cast<uint32_t>(qi) * 128u;
        const uint32_t a0 = dq.lo + static_cast<uint32_t>((qi * kTileBytes) >> 4);
        const uint32_t b0 = dk.lo + static_cast<uint32_t>((st * kTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < kHD / 16; ++kk) {
          const uint32_t koff = static_cast<uint32_t>(((kk >> 2) * kHalfTile + (kk & 3) * 32) >> 4);
          umma_ss2(d, a0 + koff, dq.hi, b0 + koff, dk.hi, kIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int qi, int st, bool first) {
        const uint32_t b0 = dv.lo + static_cast<uint32_t>((st * kTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          umma_ts2(tmem + kTmemO + static_cast<uint32_t>(qi) * 128u,
                   tmem + static_cast<uint32_t>(qi) * 128u + kk * 8, b0 + kk * (2048 >> 4), dv.hi, kIdescPV,
                   (!first || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, abort_flag);
      if (ok && n > 0) {
        ok = mbar_wait(&kv_full[0], 0, abort_flag);
        if (ok) {
          tc_fence_after();
          issue_qk(0, 0);
          tc_commit(&s_full[0]);
          if (has1) {
            issue_qk(1, 0);
            tc_commit(&s_full[1]);
          }
        }
      }
      // Fixed issue order per key tile j: P.V of query tile 0, Q.K^T of tile 0 for j+1,
      // P.V of query tile 1, Q.K^T of tile 1 for j+1.  Blocking waits (try_wait suspends
      // the thread) keep this warp off the issue slots the softmax warps share.
      for (int j = 0; ok && j < n; ++j) {
        const int st = j % kStages;
        const bool more = j + 1 < n;
        const int st1 = (j + 1) % kStages;
        if (!mbar_wait(&p_full[0], j & 1, abort_flag)) break;
        tc_fence_after();
        issue_pv(0, st, j == 0);
        if (more) {
          if (!mbar_wait(&kv_full[st1], ((j + 1) / kStages) & 1, abort_flag)) break;
          tc_fence_after();
          issue_qk(0, st1);
          tc_commit(&s_full[0]);
        }
        if (has1) {
          if (!mbar_wait(&p_full[1], j & 1, abort_flag)) break;
          tc_fence_after();
          issue_pv(1, st, j == 0);
          if (more) {
            issue_qk(1, st1);
            tc_commit(&s_full[1]);
          }
        }
        tc_commit(&kv_empty[st]);
      }
      tc_commit(o_full);
      tc_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int qi = (warp >> 2) - 1;  // query tile of this warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qt0 = q0 + qi * kBM;   // first row of this query tile
    const int qrow = qt0 + row;
    const bool active = qi == 0 || has1;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t t_s = t_lane + static_cast<uint32_t>(qi) * 128u;
    const uint32_t t_o = t_lane + kTmemO + static_cast<uint32_t>(qi) * 128u;
    const bool img_row = qrow < p.Li;
    // First invisible image key (index relative to the image keys) of this row and of the
    // tile's first row; negative when the whole image segment is in the future.
    const int row_lim = (p.gtok > 0 && img_row) ? img_keys_visible(p, q_position(p, qrow)) : INT_MAX;
    const int cta_lim = (p.gtok > 0 && qt0 < p.Li) ? img_keys_visible(p, q_position(p, qt0)) : INT_MAX;
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; active && j < n; ++j) {
      const int k0 = tr.tile(j_begin + j) * kBN;
      uint4 w4 = bits_in_smem ? reinterpret_cast<const uint4*>(sBits)[k0 >> 7]
                              : __ldg(reinterpret_cast<const uint4*>(kb_glob) + (k0 >> 7));
      const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
      if (!mbar_wait(&s_full[qi], j & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kBN];
      {
        uint32_t r[kBN];
        tmem_ld128_wait(t_s, r);
#pragma unroll
        for (int i = 0; i < kBN; ++i) s[i] = __uint_as_float(r[i]);
      }
      // Mask: visibility bits of the tile's keys, then this row's block-causal interval
      // [ca, cb) of invisible image keys.
      const bool causal_tile = (cta_lim != INT_MAX) && (k0 + kBN > p.Lh + cta_lim) &&
                               (k0 < p.Lh + p.Lik);
      if (causal_tile || (w[0] & w[1] & w[2] & w[3]) != 0xffffffffu) {
        int ca = kBN, cb = 0;
        if (row_lim != INT_MAX) {
          ca = min(max(p.Lh + row_lim - k0, 0), kBN);
          cb = min(max(p.Lh + p.Lik - k0, 0), kBN);
        }
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          const bool vis = ((w[c >> 5] >> (c & 31)) & 1u) && !(c >= ca && c < cb);
          s[c] = vis ? s[c] : -INFINITY;
        }
      }
      // Row max: 4 chains of 3-input max.
      float m4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int c = 4; c + 8 <= kBN; c += 8) {
#pragma unroll
        for (int i = 0; i < 4; ++i) m4[i] = fmax3(m4[i], s[c + 2 * i], s[c + 2 * i + 1]);
      }
      m4[0] = fmax3(m4[0], s[kBN - 4], s[kBN - 3]);
      m4[1] = fmax3(m4[1], s[kBN - 2], s[kBN - 1]);
      float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      mx *= sl2;
      const bool resc = mx > m_run + kRescaleThreshold;
      const float m_new = resc ? mx : m_run;
      const float alpha = resc ? ex2(m_run - m_new) : 1.f;
      l *= alpha;
      m_run = m_new;
      const float mref = (m_run == -INFINITY) ? 0.f : m_run;
      // P = exp2(S * scale * log2e - m) in packed-pair arithmetic: one fma.f32x2 for the
      // scaled, shifted scores of two keys, two MUFU exponentials, one bf16x2 pack and one
      // add.f32x2 into the row sum.
      float2 l2a = make_float2(0.f, 0.f), l2b = make_float2(0.f, 0.f);
      const float2 sl2x2 = make_float2(sl2, sl2);
      const float2 negm = make_float2(-mref, -mref);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int c0 = 2 * c;
          const float2 x = ffma2(make_float2(s[32 * q4 + c0], s[32 * q4 + c0 + 1]), sl2x2, negm);
          float2 e;
          if (16 * q4 + c >= kBN / 2 - 8 * kEmuPer8) {
            e = exp2_poly2(x);
          } else {
            e = make_float2(ex2(x.x), ex2(x.y));
          }
          if (c & 1) {
            l2b = fadd2(l2b, e);
          } else {
            l2a = fadd2(l2a, e);
          }
          pk[c] = kVF16 ? pack_f16x2(e.x, e.y) : pack_bf16x2(e.x, e.y);
        }
        tmem_st16(t_s + 16 * q4, pk);
      }
      l += (l2a.x + l2a.y) + (l2b.x + l2b.y);
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
        // O_i already holds every P·V of earlier tiles (the S commit this softmax waited
        // on was issued after the previous P·V of this query tile), and the next P·V
        // waits for the P-ready barrier below; rescaling after the P write keeps the S
        // registers dead here.
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t r[32];
          tmem_ld32_wait(t_o + c4 * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(t_o + c4 * 32, r);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[qi]);
    }
    if (active) {
      bool have_o = ok && n > 0 && mbar_wait(o_full, 0, abort_flag);
      have_o = __all_sync(0xffffffffu, have_o);
      tc_fence_after();
      // Every MMA has completed (or the CTA aborted and waits for nothing more), so the K ring
      // is free: 4 KB of it per softmax warp stages the epilogue's row transposes.
      uint8_t* ebuf = sK + (warp - 4) * 4096;
      const bool in_range = qrow < p.Lq;
      if (p.sc_o != nullptr) {
        // Partial of this key slice to the row's owner(s), in their (peer-mapped) buffers:
        // O / l in fp32 and the LSE (-inf when the slice saw no visible key).
        const bool seen = m_run != -INFINITY;
        const float inv_l = seen ? __frcp_rn(l) : 0.f;
        const float lse_v = seen ? (m_run * kLn2 + __logf(l)) : -INFINITY;
        const int R = p.sc_rows + (p.Lq - p.Li);
        const size_t slab = ((static_cast<size_t>(p.sc_index0 + split) * p.B + b) * p.H + h) * R;
        const bool txt_row = in_range && qrow >= p.Li;
        // a text row goes to every rank; image rows to their one owner
        const int ndest = __any_sync(0xffffffffu, txt_row) ? p.sc_ranks : 1;
        for (int d = 0; d < ndest; ++d) {
          float* dst = nullptr;
          float* dl = nullptr;
          if (in_range && (txt_row || d == 0)) {
            const int owner = txt_row ? d : qrow / p.sc_rows;
            const size_t lrow = slab + (txt_row ? p.sc_rows + (qrow - p.Li) : qrow % p.sc_rows);
            dst = p.sc_o[owner] + lrow * kHD;
            dl = p.sc_lse[owner] + lrow;
          }
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t r[32];
            if (have_o) {
              tmem_ld32_wait(t_o + c4 * 32, r);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = 0u;
            }
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * inv_l;
            warp_store_f32_rows_to(ebuf, v, dst != nullptr ? dst + c4 * 32 : nullptr, lane);
          }
          if (dl != nullptr) *dl = lse_v;
        }
      } else if (nsplit > 1) {
        // Partial result of this key slice: O / l in fp32 and its LSE (-inf when the slice
        // saw no visible key); query validity is applied by the merge.
        const bool seen = m_run != -INFINITY;  // some key of the slice is visible to this row
        const float inv_l = seen ? __frcp_rn(l) : 0.f;
        const size_t prow = ((static_cast<size_t>(split) * p.B + b) * p.H + h) * p.Lq + qrow;
        const int row0 = qt0 + quarter * 32;   // the warp's first row: its rows are contiguous
        float* wbase = p.part_o + (prow - lane) * kHD;
        const int nrows = imin(32, p.Lq - row0);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t r[32];
          if (have_o) {
            tmem_ld32_wait(t_o + c4 * 32, r);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = 0u;
          }
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * inv_l;
          warp_store_f32_rows(ebuf, v, wbase + c4 * 32, nrows, lane);
        }
        if (in_range) p.part_lse[prow] = seen ? (m_run * kLn2 + __logf(l)) : -INFINITY;
      } else if (p.acc_o != nullptr) {
        // Ring step: merge this launch's rows into the running output.
        const bool merge = (p.acc_mode & 1) != 0;
        const bool fin = (p.acc_mode & 2) != 0;
        const size_t lrow = static_cast<size_t>(bh) * p.Lq + qrow;
        const bool seen = m_run != -INFINITY;
        const float lse_b = seen ? (m_run * kLn2 + __logf(l)) : -INFINITY;
        const float lse_a = (in_range && merge) ? p.acc_lse[lrow] : -INFINITY;
        const AccWeights aw = acc_weights(lse_a, lse_b);
        const float cb = seen ? aw.wb * __frcp_rn(l) : 0.f;
        float* arow = in_range ? p.acc_o + ((static_cast<size_t>(b) * p.Lq + qrow) * p.H + h) * kHD : nullptr;
        __nv_bfloat16* dst = (in_range && fin) ? p.out_img + b * p.oi_b + (qrow / p.oi_seg) * p.oi_sseg +
                                                     (qrow % p.oi_seg) * p.oi_t + h * p.oi_h
                                               : nullptr;
        const bool read_acc = arow != nullptr && aw.wa != 0.f;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t r[32];
          if (have_o) {
            tmem_ld32_wait(t_o + c4 * 32, r);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = 0u;
          }
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * cb;
          if (read_acc) {
            const float4* s4 = reinterpret_cast<const float4*>(arow + c4 * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 a4 = s4[i];
              v[4 * i] = fmaf(aw.wa, a4.x, v[4 * i]);
              v[4 * i + 1] = fmaf(aw.wa, a4.y, v[4 * i + 1]);
              v[4 * i + 2] = fmaf(aw.wa, a4.z, v[4 * i + 2]);
              v[4 * i + 3] = fmaf(aw.wa, a4.w, v[4 * i + 3]);
            }
          }
          if (fin) {
            if (dst != nullptr) {
              uint4* d4 = reinterpret_cast<uint4*>(dst + c4 * 32);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                d4[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                                   pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
            }
          } else if (arow != nullptr) {
            float4* d4 = reinterpret_cast<float4*>(arow + c4 * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
        }
        if (in_range) {
          if (!fin) {
            p.acc_lse[lrow] = aw.lse;
          } else if (p.lse != nullptr) {
            p.lse[lrow] = aw.lse;
          }
        }
      } else {
        bool valid = in_range;
        if (in_range && p.qbits != nullptr)
          valid = (__ldg(p.qbits + static_cast<size_t>(b) * p.qwords + (qrow >> 5)) >> (qrow & 31)) & 1u;
        const bool seen = m_run != -INFINITY;
        const float inv_l = (seen && valid) ? __frcp_rn(l) : 0.f;
        __nv_bfloat16* dst = nullptr;
        if (in_range) {
          if (img_row) {
            dst = p.out_img + b * p.oi_b + (qrow / p.oi_seg) * p.oi_sseg + (qrow % p.oi_seg) * p.oi_t +
                  h * p.oi_h;
          } else {
            dst = p.out_txt + b * p.ot_b + static_cast<long long>(qrow - p.Li) * p.ot_t + h * p.ot_h;
          }
        }
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t r[32];
          if (have_o) {
            tmem_ld32_wait(t_o + c4 * 32, r);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = 0u;
          }
          uint32_t o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            o[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * inv_l, __uint_as_float(r[2 * i + 1]) * inv_l);
          warp_store_bf16_rows(ebuf, o, dst != nullptr ? dst + c4 * 32 : nullptr, lane);
        }
        if (p.lse != nullptr && in_range) {
          p.lse[static_cast<size_t>(bh) * p.Lq + qrow] =
              (seen && valid) ? (m_run * kLn2 + __logf(l)) : -INFINITY;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
  if (threadIdx.x == 0 && *abort_flag && p.status != nullptr) atomicOr(p.status, HYB_DEV_TIMEOUT);
}


// Combine the kv_splits partial results of every (batch, head, query row): LSE-weighted sum of
// the normalised partial rows, written as bf16 at the row's final position (zero for padded
// text queries), plus the final LSE when requested.  One warp per row, 4 dims per lane; a warp
// loads a row's partials (up to four slices, each LSE with its row) before any arithmetic, so
// a row costs one round trip to memory, not two (config 2: 86 -> 67.5 us per launch).
constexpr int kMergeBatch = 4;  // partial rows loaded together by the merge kernels
// A row's 128 columns are merged by 16 lanes, 8 columns (two float4) each, so a warp merges
// two rows and a lane keeps twice the bytes in flight that 32 lanes of 4 columns would (the
// merges are bound by loads in flight, not by instructions).
constexpr int kMergeLanes = 16;
constexpr int kMergeCols = kHD / kMergeLanes;     // 8
constexpr int kMergeVecs = kMergeCols / 4;        // float4 per lane and slice
constexpr int kMergeRowsPerBlock = 256 / kMergeLanes;  // 16 rows per 256-thread block

struct MergeRow {
  float m = -INFINITY;  // running maximum of the slice LSEs
  float wsum = 0.f;     // sum of exp(lse - m)
  float acc[kMergeCols] = {};
};

// Slices [s0, s0 + kMergeBatch) of row r: each LSE loaded together with its row's columns
// (one round trip per batch).  l = lane within the row's 16.
__device__ __forceinline__ void merge_load(const float* part_o, const float* part_lse, long long slice, long long r,
                                           int s0, int ns, int l, float (&lv)[kMergeBatch],
                                           float4 (&ov)[kMergeBatch][kMergeVecs]) {
#pragma unroll
  for (int u = 0; u < kMergeBatch; ++u) {
    if (s0 + u < ns) {
      lv[u] = __ldg(part_lse + (s0 + u) * slice + r);
      const float4* row = reinterpret_cast<const float4*>(part_o + ((s0 + u) * slice + r) * kHD) + l * kMergeVecs;
#pragma unroll
      for (int c = 0; c < kMergeVecs; ++c) ov[u][c] = __ldg(row + c);
    }
  }
}

// Fold slices [s0, s0 + kMergeBatch) into the running merge (the sums run in slice order; with
// at most kMergeBatch slices this is the plain LSE-weighted sum against the overall maximum).
__device__ __forceinline__ void merge_apply(const float (&lv)[kMergeBatch], const float4 (&ov)[kMergeBatch][kMergeVecs],
                                            int s0, int ns, MergeRow& st) {
  float mb = -INFINITY;
#pragma unroll
  for (int u = 0; u < kMergeBatch; ++u)
    if (s0 + u < ns) mb = fmaxf(mb, lv[u]);
  const float mn = fmaxf(st.m, mb);
  if (mn == -INFINITY) return;
  if (st.m != -INFINITY && st.m != mn) {
    const float sc = __expf(st.m - mn);
    st.wsum *= sc;
#pragma unroll
    for (int i = 0; i < kMergeCols; ++i) st.acc[i] *= sc;
  }
#pragma unroll
  for (int u = 0; u < kMergeBatch; ++u) {
    if (s0 + u < ns) {
      const float w = __expf(lv[u] - mn);
      st.wsum += w;
#pragma unroll
      for (int c = 0; c < kMergeVecs; ++c) {
        st.acc[4 * c] += w * ov[u][c].x;
        st.acc[4 * c + 1] += w * ov[u][c].y;
        st.acc[4 * c + 2] += w * ov[u][c].z;
        st.acc[4 * c + 3] += w * ov[u][c].w;
      }
    }
  }
  st.m = mn;
}

// The lane's 8 columns of a merged row, scaled, as bf16 (one 16-byte store).
__device__ __forceinline__ void merge_store_bf16(__nv_bfloat16* dst, int l, const float (&v)[kMergeCols], float sc) {
  *reinterpret_cast<uint4*>(dst + l * kMergeCols) =
      make_uint4(pack_bf16x2(v[0] * sc, v[1] * sc), pack_bf16x2(v[2] * sc, v[3] * sc),
                 pack_bf16x2(v[4] * sc, v[5] * sc), pack_bf16x2(v[6] * sc, v[7] * sc));
}

// The merged row r = (b * H + h) * Lq + qrow written out (or folded into the ring accumulator).
__device__ __forceinline__ void merge_finish(const AttnKParams& p, long long r, int b, int h, int qrow, int l,
                                             const MergeRow& st) {
  const float m = st.m, wsum = st.wsum;
  if (p.acc_o != nullptr) {
    // Ring step: the merged slices are this step's rows; fold them into the accumulator.
    const bool merge = (p.acc_mode & 1) != 0;
    const bool fin = (p.acc_mode & 2) != 0;
    const float lse_b = wsum > 0.f ? m + __logf(wsum) : -INFINITY;
    const AccWeights aw = acc_weights(merge ? p.acc_lse[r] : -INFINITY, lse_b);
    const float cb = wsum > 0.f ? aw.wb / wsum : 0.f;
    float* arow = p.acc_o + ((static_cast<size_t>(b) * p.Lq + qrow) * p.H + h) * kHD;
    float v[kMergeCols];
#pragma unroll
    for (int i = 0; i < kMergeCols; ++i) v[i] = st.acc[i] * cb;
    if (aw.wa != 0.f) {
#pragma unroll
      for (int c = 0; c < kMergeVecs; ++c) {
        const float4 a4 = reinterpret_cast<const float4*>(arow)[l * kMergeVecs + c];
        v[4 * c] = fmaf(aw.wa, a4.x, v[4 * c]);
        v[4 * c + 1] = fmaf(aw.wa, a4.y, v[4 * c + 1]);
        v[4 * c + 2] = fmaf(aw.wa, a4.z, v[4 * c + 2]);
        v[4 * c + 3] = fmaf(aw.wa, a4.w, v[4 * c + 3]);
      }
    }
    if (fin) {
      __nv_bfloat16* dst = p.out_img + b * p.oi_b + (qrow / p.oi_seg) * p.oi_sseg + (qrow % p.oi_seg) * p.oi_t +
                           h * p.oi_h;
      merge_store_bf16(dst, l, v, 1.f);
      if (p.lse != nullptr && l == 0) p.lse[r] = aw.lse;
    } else {
#pragma unroll
      for (int c = 0; c < kMergeVecs; ++c)
        reinterpret_cast<float4*>(arow)[l * kMergeVecs + c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
      if (l == 0) p.acc_lse[r] = aw.lse;
    }
    return;
  }
  bool valid = true;
  if (p.qbits != nullptr)
    valid = (__ldg(p.qbits + static_cast<size_t>(b) * p.qwords + (qrow >> 5)) >> (qrow & 31)) & 1u;
  const float inv = (wsum > 0.f && valid) ? 1.f / wsum : 0.f;
  __nv_bfloat16* dst = qrow < p.Li
                           ? p.out_img + b * p.oi_b + (qrow / p.oi_seg) * p.oi_sseg + (qrow % p.oi_seg) * p.oi_t +
                                 h * p.oi_h
                           : p.out_txt + b * p.ot_b + static_cast<long long>(qrow - p.Li) * p.ot_t + h * p.ot_h;
  merge_store_bf16(dst, l, st.acc, inv);
  if (p.lse != nullptr && l == 0) p.lse[r] = (wsum > 0.f && valid) ? (m + __logf(wsum)) : -INFINITY;
}

// 16 lanes per query row: blockIdx.y = b * H + h, the block's 16 rows [16 blockIdx.x, + 16) lie
// in one query pair (16 divides the pair's 256 rows), so a block of an unsplit pair (whose rows
// the attention kernel wrote itself) leaves at once.  No index division per row.
__global__ void __launch_bounds__(256, 4) merge_splits_kernel(const AttnKParams p,
                                                          const __grid_constant__ UnitMap um) {
  const int q_first = static_cast<int>(blockIdx.x) * kMergeRowsPerBlock;
  const int ns = splits_of_pair(um, um.npairs - 1 - q_first / kPairRows);
  if (ns <= 1) return;
  const int qrow = q_first + static_cast<int>(threadIdx.x) / kMergeLanes;
  if (qrow >= p.Lq) return;
  const int l = threadIdx.x & (kMergeLanes - 1);
  const int bh = static_cast<int>(blockIdx.y);
  const long long slice = static_cast<long long>(p.B) * p.H * p.Lq;
  const long long r = static_cast<long long>(bh) * p.Lq + qrow;
  float lv[kMergeBatch];
  float4 ov[kMergeBatch][kMergeVecs];
  MergeRow st;
  for (int s0 = 0; s0 < ns; s0 += kMergeBatch) {
    merge_load(p.part_o, p.part_lse, slice, r, s0, ns, l, lv, ov);
    merge_apply(lv, ov, s0, ns, st);
  }
  merge_finish(p, r, bh / p.H, bh % p.H, qrow, l, st);
}

// Owner side of a partial scatter: one warp per (batch, head, row) of this rank's buffers, the
// lane's four columns of the `count` partials merged by log-sum-exp (the merge of
// dynamic_ring_attention.py:86-105 over all partials at once).
struct MergePartialsParams {
  int count, B, H, rows, txt;
  const float* o;
  const float* lse;
  __nv_bfloat16* out_img;
  long long oi_b, oi_t, oi_h;
  __nv_bfloat16* out_txt;
  long long ot_b, ot_t, ot_h;
  const uint8_t* text_mask;
  long long tm_sb;
  float* lse_out;
};

// One warp per row: blockIdx.y = b * H + h, rows [8 blockIdx.x, + 8) of the owner's R rows.
__global__ void __launch_bounds__(256) merge_partials_kernel(const MergePartialsParams p) {
  const int R = p.rows + p.txt;
  const long long slice = static_cast<long long>(p.B) * p.H * R;  // elements between partial indices
  const int l = threadIdx.x & (kMergeLanes - 1);
  const int lr = static_cast<int>(blockIdx.x) * kMergeRowsPerBlock + static_cast<int>(threadIdx.x) / kMergeLanes;
  if (lr < R) {
    const int bh = static_cast<int>(blockIdx.y);
    const int h = bh % p.H;
    const int b = bh / p.H;
    const long long r = static_cast<long long>(bh) * R + lr;
    // four partials at a time, each LSE loaded with its row (one round trip per four)
    float lv[kMergeBatch];
    float4 ov[kMergeBatch][kMergeVecs];
    MergeRow st;
    for (int s0 = 0; s0 < p.count; s0 += kMergeBatch) {
      merge_load(p.o, p.lse, slice, r, s0, p.count, l, lv, ov);
      merge_apply(lv, ov, s0, p.count, st);
    }
    const float m = st.m, wsum = st.wsum;
    const bool img = lr < p.rows;
    const bool valid = img || p.text_mask == nullptr || p.text_mask[b * p.tm_sb + (lr - p.rows)] != 0;
    const float inv = (wsum > 0.f && valid) ? 1.f / wsum : 0.f;
    __nv_bfloat16* dst = img ? p.out_img + b * p.oi_b + static_cast<long long>(lr) * p.oi_t + h * p.oi_h
                             : p.out_txt + b * p.ot_b + static_cast<long long>(lr - p.rows) * p.ot_t + h * p.ot_h;
    merge_store_bf16(dst, l, st.acc, inv);
    if (p.lse_out != nullptr && l == 0) p.lse_out[r] = (wsum > 0.f && valid) ? m + __logf(wsum) : -INFINITY;
  }
}

// ------------------------------------------------------------------ staging kernels
struct StageSeg {
  const int* rows;  // token -> source row map (history ring), or null
  const void* data;
  const float* scale;
  long long s_b, s_t, s_h, c_b, c_t, c_h;
  int fmt;
  int len;
  int bcast;  // 1: batch index 0 for every output batch
};

struct StageParams {
  int B, H, L, nout, nseg;
  long long out_pitch;  // rows between consecutive (batch, head) slabs of out (0: L)
  int out_t0;           // row t goes to row out_t0 + t of its slab
  StageSeg seg[2][3];
  void* out[2];       // [B, H, L, 128]
  int out_f16[2];     // 1: output in fp16 (the P.V operand), 0: bf16.  Either way a value is the
                      // bf16 the reference decodes (dequantize_kv rounds code * scale to bf16):
                      // fp16 holds every such bf16 value exactly in the range of K/V activations
};

// Sixteen consecutive values [16 lane8, 16 lane8 + 16) of one (batch, token, head) row as
// fp32: bf16 sources exactly, quantised sources as code * scale (one fp32 multiply, as
// dequantize_kv does before its single rounding).  Codes
// are read as two 8-byte loads: a quantised view guarantees 8-byte, not 16-byte, rows.
__device__ __forceinline__ void load_row16(const StageSeg& s, int b, int t, int h, int lane8, float (&v)[16]) {
  const int bb = s.bcast ? 0 : b;
  if (s.rows != nullptr) t = __ldg(s.rows + t);
  if (s.fmt == HYB_FMT_BF16) {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(s.data) + bb * s.s_b +
                                                      t * s.s_t + h * s.s_h + lane8 * 16);
    const uint4 raw[2] = {src[0], src[1]};
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 f = __bfloat1622float2(p2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
    return;
  }
  const float sc = s.scale[bb * s.c_b + t * s.c_t + h * s.c_h];
  const uint2* src = reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(s.data) + bb * s.s_b + t * s.s_t +
                                                    h * s.s_h + lane8 * 16);
  const uint2 raw[2] = {src[0], src[1]};
  const uint8_t* by = reinterpret_cast<const uint8_t*>(raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float a, c;
    if (s.fmt == HYB_FMT_INT8) {
      a = static_cast<float>(static_cast<int8_t>(by[2 * i]));
      c = static_cast<float>(static_cast<int8_t>(by[2 * i + 1]));
    } else {
      const __nv_fp8x2_storage_t pair = static_cast<__nv_fp8x2_storage_t>(by[2 * i] | (by[2 * i + 1] << 8));
      const float2 f = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3)));
      a = f.x;
      c = f.y;
    }
    v[2 * i] = __fmul_rn(a, sc);
    v[2 * i + 1] = __fmul_rn(c, sc);
  }
}

// One 8-lane group per (batch, token, head) row in source order (head fastest, so the reads
// of consecutive groups are contiguous across heads), 16 values per lane.  A group's
// (b, t, h) is decomposed once and then advanced by the grid stride with carries, not
// recomputed by 64-bit division per row (the division chain made the earlier 16-lane form
// issue-bound).  Output head-major [B, H, L, 128]; the launcher checks B * L * H * 8 < 2^31.
__global__ void __launch_bounds__(256) stage_kernel(const StageParams p) {
  const int Ls = p.L;
  const int lane8 = threadIdx.x & 7;
  const int g = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 3);
  const int step = static_cast<int>((gridDim.x * blockDim.x) >> 3);
  int h = g % p.H;
  int t = (g / p.H) % Ls;
  int b = (g / p.H) / Ls;
  const int dh = step % p.H;
  const int dt = (step / p.H) % Ls;
  const int db = (step / p.H) / Ls;
  while (b < p.B) {
    int ts = t, si = 0;  // position within segment si
    while (si < p.nseg - 1 && ts >= p.seg[0][si].len) {
      ts -= p.seg[0][si].len;
      ++si;
    }
    const long long out_off = ((static_cast<long long>(b) * p.H + h) * p.out_pitch + p.out_t0 + t) * kHD + lane8 * 16;
#pragma unroll
    for (int o = 0; o < 2; ++o) {
      if (o < p.nout) {
        float v[16];
        load_row16(p.seg[o][si], b, ts, h, lane8, v);
        uint4 packed[2];
        uint32_t* w = reinterpret_cast<uint32_t*>(packed);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          w[i] = p.out_f16[o] ? pack_f16x2(bf16_round(v[2 * i]), bf16_round(v[2 * i + 1]))
                              : pack_bf16x2(v[2 * i], v[2 * i + 1]);
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out[o]) + out_off);
        dst[0] = packed[0];
        dst[1] = packed[1];
      }
    }
    h += dh;
    int carry = 0;
    if (h >= p.H) {
      h -= p.H;
      carry = 1;
    }
    t += dt + carry;
    carry = 0;
    if (t >= Ls) {
      t -= Ls;
      carry = 1;
    }
    b += db + carry;
  }
}

// Sequence-parallel K/V blocks -> one head-major bf16 K/V of the whole sequence.  Position
// `pos` lies in chunk c ([bounds[c], bounds[c+1])), held by rank owner[c] at block row
// row0[c] + (pos - bounds[c]).  A block is [K codes | V codes | K scales | V scales] for Lmax
// rows of H heads (the ring message layout); decode as load_row16.
constexpr int kMaxGatherChunks = 128;
struct GatherParams {
  int L, H, Lmax, fmt, nchunks;
  int v_f16;  // 1: V written in fp16 (the bf16 decode, converted exactly) for a P.V in fp16
  const uint8_t* blocks[64];
  int bounds[kMaxGatherChunks + 1];
  int owner[kMaxGatherChunks];
  int row0[kMaxGatherChunks];
  __nv_bfloat16* out_k;
  __nv_bfloat16* out_v;
};

// One 8-lane group per (head, position) row, 16 values per lane, positions fastest (the
// head-major output rows are written in order); (h, pos) advanced by the grid stride with a
// carry instead of a 64-bit division per row.  The launcher checks H * L * 8 < 2^31.
__global__ void __launch_bounds__(256) gather_stage_kernel(const GatherParams p) {
  const long long codes = static_cast<long long>(p.Lmax) * p.H * kHD;
  const int lane8 = threadIdx.x & 7;
  const int g = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 3);
  const int step = static_cast<int>((gridDim.x * blockDim.x) >> 3);
  int pos = g % p.L;
  int h = g / p.L;
  const int dpos = step % p.L;
  const int dh = step / p.L;
  while (h < p.H) {
    int lo = 0, hi = p.nchunks - 1;  // chunk containing pos
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.bounds[mid] <= pos) {
        lo = mid;
      } else {
        hi = mid - 1;
      }
    }
    const uint8_t* blk = p.blocks[p.owner[lo]];
    const int row = p.row0[lo] + (pos - p.bounds[lo]);
    const long long out_off = (static_cast<long long>(h) * p.L + pos) * kHD + lane8 * 16;
#pragma unroll
    for (int o = 0; o < 2; ++o) {
      StageSeg sg;
      sg.rows = nullptr;
      sg.data = blk + o * codes;
      sg.scale = reinterpret_cast<const float*>(blk + 2 * codes) + o * static_cast<long long>(p.Lmax) * p.H;
      sg.s_b = 0;
      sg.s_t = static_cast<long long>(p.H) * kHD;
      sg.s_h = kHD;
      sg.c_b = 0;
      sg.c_t = p.H;
      sg.c_h = 1;
      sg.fmt = p.fmt;
      sg.len = p.Lmax;
      sg.bcast = 0;
      float v[16];
      load_row16(sg, 0, row, h, lane8, v);
      uint4 packed[2];
      uint32_t* w = reinterpret_cast<uint32_t*>(packed);
      const bool f16 = o == 1 && p.v_f16;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        w[i] = f16 ? pack_f16x2(bf16_round(v[2 * i]), bf16_round(v[2 * i + 1])) : pack_bf16x2(v[2 * i], v[2 * i + 1]);
      uint4* dst = reinterpret_cast<uint4*>((o == 0 ? p.out_k : p.out_v) + out_off);
      dst[0] = packed[0];
      dst[1] = packed[1];
    }
    pos += dpos;
    int carry = 0;
    if (pos >= p.L) {
      pos -= p.L;
      carry = 1;
    }
    h += dh + carry;
  }
}

// Visibility bitmap with the first Lk keys of every batch row set (ring blocks: every key
// of the block is valid; the block-causal rule is applied by the attention kernel).
__global__ void __launch_bounds__(256) key_bits_kernel(int B, int Lk, int kwords, uint32_t* bits) {
  const long long n = static_cast<long long>(B) * kwords;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int w = static_cast<int>(i % kwords);
    const int lo = w * 32;
    uint32_t word = 0u;
    if (Lk >= lo + 32) {
      word = 0xffffffffu;
    } else if (Lk > lo) {
      word = (1u << (Lk - lo)) - 1u;
    }
    bits[i] = word;
  }
}

struct MaskParams {
  int B, Lh, Li, Lik, Lt, Lk, kwords, Lq, qwords, attend_txt;  // Li image queries, Lik image keys
  const int* hist_rows;
  const uint8_t* cache_mask;
  long long cm_sb;
  int cm_bcast;
  const uint8_t* text_mask;
  long long tm_sb;
  uint32_t* kbits;
  uint32_t* qbits;
};

__global__ void __launch_bounds__(256) mask_kernel(const MaskParams p) {
  const long long kw_total = static_cast<long long>(p.B) * p.kwords;
  const long long qw_total = static_cast<long long>(p.B) * p.qwords;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       i < kw_total + qw_total; i += static_cast<long long>(gridDim.x) * blockDim.x) {
    uint32_t word = 0;
    if (i < kw_total) {
      const int b = static_cast<int>(i / p.kwords);
      const int w = static_cast<int>(i % p.kwords);
      for (int bit = 0; bit < 32; ++bit) {
        const int k = w * 32 + bit;
        bool vis;
        if (k < p.Lh) {
          const int row = p.hist_rows != nullptr ? p.hist_rows[k] : k;
          vis = p.cache_mask == nullptr || p.cache_mask[(p.cm_bcast ? 0 : b) * p.cm_sb + row] != 0;
        } else if (k < p.Lh + p.Lik) {
          vis = true;
        } else if (k < p.Lk) {
          vis = p.text_mask == nullptr || p.text_mask[b * p.tm_sb + (k - p.Lh - p.Lik)] != 0;
        } else {
          vis = false;
        }
        word |= (vis ? 1u : 0u) << bit;
      }
      p.kbits[i] = word;
    } else {
      const long long j = i - kw_total;
      const int b = static_cast<int>(j / p.qwords);
      const int w = static_cast<int>(j % p.qwords);
      for (int bit = 0; bit < 32; ++bit) {
        const int q = w * 32 + bit;
        bool vis;
        if (q < p.Li) {
          vis = true;
        } else if (q < p.Lq) {
          vis = p.text_mask == nullptr || p.text_mask[b * p.tm_sb + (q - p.Li)] != 0;
        } else {
          vis = false;
        }
        word |= (vis ? 1u : 0u) << bit;
      }
      p.qbits[j] = word;
    }
  }
}

// ------------------------------------------------------------------ host helpers
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [BH, L, 128] 16-bit head-major tensor (bf16 or f16), 64 x 128 boxes with 128-byte swizzle.
// [BH, L, 128] rows of 16-bit values, `pitch` rows (>= L; 0: L) between consecutive bh slabs.
int make_map(CUtensorMap* map, const void* base, int BH, int L, bool f16 = false, long long pitch = 0) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(HYB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (pitch <= 0) pitch = L;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHD), static_cast<cuuint64_t>(L), static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHD) * 2, static_cast<cuuint64_t>(pitch) * kHD * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HYB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return HYB_OK;
}

int grid_for(long long items, int threads) {
  long long blocks = (items + threads - 1) / threads;
  const long long cap = 148LL * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int device_sm_count();

// Blocks of 256 threads for `lanes` work lanes of a grid-striding kernel: at most one
// resident wave (blocks per SM from the occupancy calculator, cached per kernel in *per_sm).
template <typename K>
long long wave_blocks(K kernel, int* per_sm, long long lanes) {
  if (*per_sm == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, 256, 0) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 4;
    }
    *per_sm = n;
  }
  long long blocks = (lanes + 255) / 256;
  const long long wave = static_cast<long long>(device_sm_count()) * *per_sm;
  return blocks > wave ? wave : (blocks < 1 ? 1 : blocks);
}

// stage_kernel, 8 lanes per (batch, token, head) row.
int launch_stage(StageParams sp, cudaStream_t stream) {
  const long long lanes = static_cast<long long>(sp.B) * sp.L * sp.H * 8;
  if (lanes <= 0) return HYB_OK;
  if (sp.out_pitch == 0) sp.out_pitch = sp.L;
  if (lanes >= (1LL << 31)) return fail(HYB_ERR_UNSUPPORTED, "stage: %lld rows exceed the 32-bit row index", lanes / 8);
  static int per_sm = 0;
  stage_kernel<<<static_cast<unsigned>(wave_blocks(stage_kernel, &per_sm, lanes)), 256, 0, stream>>>(sp);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

int check_view(const hyb_tensor4& v, const char* name, bool allow_quant) {
  if (v.data == nullptr) return fail(HYB_ERR_INVALID_ARG, "%s: null data", name);
  if (v.fmt == HYB_FMT_BF16) {
    if (!al16(v.data) || (v.s_b % 8) || (v.s_t % 8) || (v.s_h % 8))
      return fail(HYB_ERR_INVALID_ARG, "%s: bf16 rows must be 16-byte aligned", name);
    return HYB_OK;
  }
  if (!allow_quant || (v.fmt != HYB_FMT_E4M3 && v.fmt != HYB_FMT_INT8))
    return fail(HYB_ERR_UNSUPPORTED, "%s: unsupported format %d", name, v.fmt);
  if ((reinterpret_cast<uintptr_t>(v.data) & 7u) || (v.s_b % 8) || (v.s_t % 8) || (v.s_h % 8))
    return fail(HYB_ERR_INVALID_ARG, "%s: code rows must be 8-byte aligned", name);
  if (v.scale == nullptr) return fail(HYB_ERR_INVALID_ARG, "%s: quantised view without scale", name);
  return HYB_OK;
}

StageSeg seg_of(const hyb_tensor4& v, int len, int bcast, const int* rows = nullptr) {
  StageSeg s;
  s.rows = rows;
  s.data = v.data;
  s.scale = v.scale;
  s.s_b = v.s_b;
  s.s_t = v.s_t;
  s.s_h = v.s_h;
  s.c_b = v.ss_b;
  s.c_t = v.ss_t;
  s.c_h = v.ss_h;
  s.fmt = v.fmt;
  s.len = len;
  s.bcast = bcast;
  return s;
}

long long align256(long long x) { return (x + 255) & ~255LL; }

struct WorkspaceLayout {
  long long q, k, v, kbits, qbits, part_o, part_lse, total;
  int Lq, Lk, kwords, qwords, kv_splits;
};

// Multiprocessor count of the current device (148 on B200; 148 when no device is visible).
int device_sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 148;
  }
  return n;
}

// Key-slice count per query pair.  One pair-CTA per (pair, head, batch) leaves the last wave
// of CTAs partly empty; slicing the key range multiplies the CTAs by S at the price of
// writing and re-reading fp32 partial rows.  Estimated time: attention at ~1 PFLOP/s scaled
// by the wave quantisation ceil(c S / sms) / (c S / sms), plus the partial traffic at ~6 TB/s
// and a merge launch.  HYB_KV_SPLITS overrides (1..16).
int choose_kv_splits(int B, int H, int Lq, int Lk, int sms) {
  const char* e = getenv("HYB_KV_SPLITS");
  if (e != nullptr) {
    const int v = atoi(e);
    if (v >= 1 && v <= 16) return v;
  }
  const long long ctas = static_cast<long long>((Lq + kPairRows - 1) / kPairRows) * H * B;
  const int tiles = (Lk + kBN - 1) / kBN;
  if (ctas <= 0 || tiles <= 0) return 1;
  const double attn_us = 4.0 * 128.0 * H * B * static_cast<double>(Lq) * Lk / 1e15 * 1e6 * 0.75;
  const double rows = static_cast<double>(B) * H * Lq;
  int best = 1;
  double best_t = 1e300;
  for (int sp = 1; sp <= 16; ++sp) {
    if (sp > 1 && tiles / sp < 16) break;  // keep at least 16 key tiles per slice
    const double w = static_cast<double>(ctas) * sp / sms;
    const double t = attn_us * std::ceil(w) / w + (sp > 1 ? sp * rows * 1032.0 / 6e12 * 1e6 + 5.0 : 0.0);
    if (t < best_t * 0.98) {
      best_t = t;
      best = sp;
    }
  }
  return best;
}

// Capacity of the partial buffers: the most key slices any query pair may be cut into (the
// per-pair counts are chosen at launch by plan_units).  The dense estimate above, raised to 4
// when the launch has fewer than 8 waves of pair-CTAs (its tail is then a large share), and
// bounded to 1 GiB of partial rows.  (Room for more slices was measured slower at 3 heads:
// the planner then cut pairs into 7-8 slices, whose partial rows cost more than it models.)
int split_capacity(int B, int H, int Lq, int Lk, int sms) {
  const char* e = getenv("HYB_KV_SPLITS");
  if (e != nullptr) {
    const int v = atoi(e);
    if (v >= 1 && v <= 16) return v;
  }
  const long long ctas = static_cast<long long>((Lq + kPairRows - 1) / kPairRows) * H * B;
  const int tiles = (Lk + kBN - 1) / kBN;
  if (ctas <= 0 || tiles < 32) return 1;
  int cap = choose_kv_splits(B, H, Lq, Lk, sms);
  if (ctas < 8LL * sms) cap = imax(cap, 4);
  cap = imin(cap, imax(1, tiles / 8));
  while (cap > 1 && static_cast<long long>(cap) * B * H * Lq * (kHD * 4 + 4) > (1LL << 30)) --cap;
  return cap;
}

// Per-pair key-slice counts of one launch, chosen by simulating the in-order dispatch of the
// work list onto the SMs: a unit costs its key tiles plus a fixed ~2 tiles (tensor-memory
// setup, Q load, epilogue); a split pair adds its fp32 partial rows written and merged at
// ~6 TB/s and the merge launch.  Candidate slice lengths U give k_i = ceil(n_i / U) <= cap.
// Plans are cached per launch geometry.
struct PlanKey {
  long long v[17];
  bool operator<(const PlanKey& o) const {
    for (int i = 0; i < 17; ++i)
      if (v[i] != o.v[i]) return v[i] < o.v[i];
    return false;
  }
};
std::mutex g_plan_mu;
std::map<PlanKey, UnitMap> g_plans;

UnitMap plan_units(const AttnKParams& kp, int cap, int sms) {
  UnitMap um;
  memset(&um, 0, sizeof(um));
  const int np = (kp.num_qtiles + 1) / 2;
  um.npairs = np;
  cap = imax(cap, 1);
  const char* e = getenv("HYB_KV_SPLITS");
  const int forced = e != nullptr ? atoi(e) : 0;
  int uniform = 0;
  if (kp.sc_o != nullptr) {
    uniform = cap;  // every pair cut into exactly the scatter's slice count
  } else if (forced >= 1) {
    uniform = imin(forced, cap);
  } else if (cap <= 1) {
    uniform = 1;
  } else if (np > kMaxPairTab) {
    uniform = imin(cap, choose_kv_splits(kp.B, kp.H, kp.Lq, kp.Lk, sms));
  }
  if (uniform > 0 || np == 0) {
    um.uniform = imax(uniform, 1);
    um.per_bh = np * um.uniform;
    um.max_k = um.uniform;
    return um;
  }
  const PlanKey key = {{kp.B, kp.H, kp.Lq, kp.Lk, kp.Lh, kp.Li, kp.Lik, kp.gtok, kp.q_pos0, kp.k_pos0, kp.q_seg,
                        kp.q_pos1, kp.k_seg, kp.k_pos1, cap, sms, 1}};
  {
    std::lock_guard<std::mutex> lock(g_plan_mu);
    auto it = g_plans.find(key);
    if (it != g_plans.end()) return it->second;
  }
  std::vector<int> n(np), rows(np);
  int nmax = 0;
  long long total = 0;
  for (int i = 0; i < np; ++i) {
    const int qp = np - 1 - i;
    n[i] = key_tiles(kp, qp * kPairRows, kPairRows).count();
    rows[i] = imin(kPairRows, kp.Lq - qp * kPairRows);
    nmax = imax(nmax, n[i]);
    total += n[i];
  }
  const int BH = kp.B * kp.H;
  std::vector<int> cands;
  for (int sp = 1; sp <= cap; ++sp) cands.push_back(imax(1, (nmax + sp - 1) / sp));
  for (int w = 1; w <= 64; ++w) {
    const long long u = (total * BH + static_cast<long long>(w) * sms - 1) / (static_cast<long long>(w) * sms);
    if (u >= 4 && u < nmax) cands.push_back(static_cast<int>(u));
  }
  // Second family: a total of M units per (b, h) aimed at whole waves, slices handed to the
  // pairs in proportion to their tiles (k_i = round(n_i M / sum n)).
  std::vector<int> totals;
  for (int w = 1; w <= 64; ++w) {
    const long long m = (static_cast<long long>(w) * sms) / BH;
    for (long long d = -1; d <= 0; ++d)
      if (m + d >= np && m + d <= static_cast<long long>(np) * cap) totals.push_back(static_cast<int>(m + d));
  }
  const int n_cands = static_cast<int>(cands.size());
  const double c_fix = 2.0;
  const double t_tile = 2.0e-6;
  double best_t = 1e300;
  std::vector<int> best_k(np, 1), k(np);
  for (int c = 0; c < n_cands + static_cast<int>(totals.size()); ++c) {
    bool any_split = false;
    double over = 0.0;
    for (int i = 0; i < np; ++i) {
      if (c < n_cands) {
        const int U = cands[c];
        k[i] = imin(cap, imax(1, (n[i] + U - 1) / U));
      } else {
        const double share = total > 0 ? static_cast<double>(n[i]) * totals[c - n_cands] / total : 1.0;
        k[i] = imin(cap, imax(1, static_cast<int>(share + 0.5)));
      }
      if (k[i] > 1) {
        any_split = true;
        over += static_cast<double>(rows[i]) * BH * k[i] * (kHD * 4 + 4) * 2.0 / 6e12 / t_tile;
      }
    }
    if (any_split) over += 2.0;
    std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
    for (int sm = 0; sm < sms; ++sm) free_at.push(0.0);
    double makespan = 0.0;
    for (int bh = 0; bh < BH; ++bh) {
      for (int i = 0; i < np; ++i) {
        for (int kk = 0; kk < k[i]; ++kk) {
          const long long len = (static_cast<long long>(n[i]) * (kk + 1)) / k[i] - (static_cast<long long>(n[i]) * kk) / k[i];
          const double t = free_at.top() + static_cast<double>(len) + c_fix;
          free_at.pop();
          free_at.push(t);
          if (t > makespan) makespan = t;
        }
      }
    }
    const double t = makespan + over;
    if (t < best_t * 0.99) {
      best_t = t;
      best_k = k;
    }
  }
  um.prefix[0] = 0;
  um.max_k = 1;
  for (int i = 0; i < np; ++i) {
    um.prefix[i + 1] = um.prefix[i] + best_k[i];
    um.max_k = imax(um.max_k, best_k[i]);
  }
  um.per_bh = um.prefix[np];
  um.uniform = 0;
  std::lock_guard<std::mutex> lock(g_plan_mu);
  if (g_plans.size() > 1024) g_plans.clear();
  g_plans[key] = um;
  return um;
}

WorkspaceLayout layout_for(int B, int H, int Lh, int Li, int Lik, int Lt, int attend_txt, int sms,
                           bool staged = false) {
  WorkspaceLayout w;
  w.Lq = Li + Lt;
  w.Lk = Lh + Lik + (attend_txt ? Lt : 0);
  w.kwords = ((w.Lk + kBN - 1) / kBN) * (kBN / 32);
  w.qwords = (w.Lq + 31) / 32;
  long long off = 0;
  w.q = off;
  off = align256(off + static_cast<long long>(B) * H * w.Lq * kHD * 2);
  // (a call with pre-decoded history stages its keys into the caller's buffers)
  const long long kv_rows = staged ? 0 : static_cast<long long>(B) * H * w.Lk;
  w.k = off;
  off = align256(off + kv_rows * kHD * 2);
  w.v = off;
  off = align256(off + kv_rows * kHD * 2);
  w.kbits = off;
  off = align256(off + static_cast<long long>(B) * w.kwords * 4);
  w.qbits = off;
  off = align256(off + static_cast<long long>(B) * (w.qwords > 0 ? w.qwords : 1) * 4);
  w.kv_splits = split_capacity(B, H, w.Lq, w.Lk, sms);
  w.part_o = off;
  w.part_lse = off;
  if (w.kv_splits > 1) {
    off = align256(off + static_cast<long long>(w.kv_splits) * B * H * w.Lq * kHD * 4);
    w.part_lse = off;
    off = align256(off + static_cast<long long>(w.kv_splits) * B * H * w.Lq * 4);
  }
  w.total = off;
  return w;
}

template <int kEmuPer8, bool kVF16>
int launch_attn2_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnKParams& kp,
                   const UnitMap& um, cudaStream_t stream) {
  const int smem = 1024 + kTileBytes * (2 + 2 * kStages) + 256 + kMaxSmemBitWords * 4;
  static bool attr_set = false;
  if (!attr_set) {
    HYB_CUDA_TRY(cudaFuncSetAttribute(attn_fwd2_kernel<kEmuPer8, kVF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      smem));
    attr_set = true;
  }
  const long long units = static_cast<long long>(kp.B) * kp.H * um.per_bh;
  if (units <= 0 || units > INT_MAX) return fail(HYB_ERR_UNSUPPORTED, "attention: %lld work units", units);
  attn_fwd2_kernel<kEmuPer8, kVF16><<<static_cast<unsigned>(units), kThreads2, smem, stream>>>(mq, mk, mv, kp, um);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

// Share of exponentials computed on the FMA pipe, in eighths of the score pairs: 0 unless
// HYB_EXP_EMU selects 2 or more (built variants: none, a quarter).
int exp_emu_per8() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("HYB_EXP_EMU");
    v = (e != nullptr && e[0] >= '0' && e[0] <= '4') ? (e[0] - '0') : 0;
  }
  return v;
}

int launch_attn2(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnKParams& kp,
                 const UnitMap& um, bool v_f16, cudaStream_t stream) {
  // Exponentials on the FMA pipe: none by default (measured fastest); HYB_EXP_EMU=2 gives a
  // quarter of every row's pairs.
  const bool emu = exp_emu_per8() >= 2;
  if (v_f16) return emu ? launch_attn2_t<2, true>(mq, mk, mv, kp, um, stream) : launch_attn2_t<0, true>(mq, mk, mv, kp, um, stream);
  return emu ? launch_attn2_t<2, false>(mq, mk, mv, kp, um, stream) : launch_attn2_t<0, false>(mq, mk, mv, kp, um, stream);
}

// Validate the arguments and translate them into kernel parameters (no device access).
int fill_params(const hyb_attn_args* a, AttnKParams& kp) {
  memset(&kp, 0, sizeof(kp));
  if (a->D != kHD) return fail(HYB_ERR_UNSUPPORTED, "attention: head_dim %d != 128", a->D);
  const int Lik = a->img_k_len > 0 ? a->img_k_len : a->img_len;
  if (a->B <= 0 || a->H <= 0 || a->Lq < 0 || a->Lk < 0 || a->hist_len < 0 || a->img_len < 0 ||
      a->img_k_len < 0 || a->hist_len + Lik > a->Lk || a->img_len > a->Lq || a->group_tokens < 0)
    return fail(HYB_ERR_INVALID_ARG, "attention: inconsistent sizes");
  const bool two_q = a->q_seg > 0 && a->q_seg < a->img_len;
  const bool two_k = a->k_seg > 0 && a->k_seg < Lik;
  if ((two_q && static_cast<long long>(a->q_pos1) < static_cast<long long>(a->q_pos0) + a->q_seg) ||
      (two_k && static_cast<long long>(a->k_pos1) < static_cast<long long>(a->k_pos0) + a->k_seg) ||
      a->q_pos0 < 0 || a->k_pos0 < 0 || (two_q && a->q_pos1 < 0) || (two_k && a->k_pos1 < 0))
    return fail(HYB_ERR_INVALID_ARG, "attention: position segments must be nonnegative and increasing");
  if (a->acc_o != nullptr &&
      (a->acc_lse == nullptr || !al16(a->acc_o) || a->Lq != a->img_len || a->acc_mode < 0 || a->acc_mode > 3))
    return fail(HYB_ERR_INVALID_ARG,
                "attention: the ring accumulator needs acc_lse, 16-byte alignment, image queries only, mode 0..3");
  if (a->Lq == 0) return HYB_OK;
  if (!al16(a->q) || !al16(a->k) || !al16(a->v)) return fail(HYB_ERR_INVALID_ARG, "attention: q/k/v misaligned");
  if (a->kwords < ((a->Lk + kBN - 1) / kBN) * (kBN / 32) || (a->kwords % 4) != 0 || !al16(a->kbits))
    return fail(HYB_ERR_INVALID_ARG, "attention: kbits must hold 4 aligned words per key tile");
  if (a->img_len > 0 && a->scatter == nullptr) {  // a partial scatter writes no final rows here
    if (a->out_img == nullptr || !al16(a->out_img) || (a->oi_sb % 8) || (a->oi_st % 8) || (a->oi_sh % 8) ||
        (a->oi_sseg % 8) || a->oi_seg <= 0)
      return fail(HYB_ERR_INVALID_ARG, "attention: image output misaligned");
  }
  if (a->Lq > a->img_len && a->scatter == nullptr) {
    if (a->out_txt == nullptr || !al16(a->out_txt) || (a->ot_sb % 8) || (a->ot_st % 8) || (a->ot_sh % 8))
      return fail(HYB_ERR_INVALID_ARG, "attention: text output misaligned");
  }
  kp.B = a->B;
  kp.H = a->H;
  kp.Lq = a->Lq;
  kp.Lk = a->Lk;
  kp.Lh = a->hist_len;
  kp.Li = a->img_len;
  kp.Lik = Lik;
  kp.gtok = a->group_tokens;
  kp.q_pos0 = a->q_pos0;
  kp.k_pos0 = a->k_pos0;
  kp.q_seg = two_q ? a->q_seg : a->img_len;
  kp.q_pos1 = two_q ? a->q_pos1 : 0;
  kp.k_seg = two_k ? a->k_seg : Lik;
  kp.k_pos1 = two_k ? a->k_pos1 : 0;
  kp.acc_o = a->acc_o;
  kp.acc_lse = a->acc_lse;
  kp.acc_mode = a->acc_mode;
  const float scale = a->softmax_scale > 0.f ? a->softmax_scale : 1.0f / sqrtf(static_cast<float>(kHD));
  kp.scale_log2 = scale * kLog2e;
  kp.kbits = a->kbits;
  kp.kwords = a->kwords;
  kp.qbits = a->qbits;
  kp.qwords = a->qwords;
  kp.out_img = static_cast<__nv_bfloat16*>(a->out_img);
  kp.oi_b = a->oi_sb;
  kp.oi_t = a->oi_st;
  kp.oi_h = a->oi_sh;
  kp.oi_seg = a->oi_seg > 0 ? a->oi_seg : 1;
  kp.oi_sseg = a->oi_sseg;
  kp.out_txt = static_cast<__nv_bfloat16*>(a->out_txt);
  kp.ot_b = a->ot_sb;
  kp.ot_t = a->ot_st;
  kp.ot_h = a->ot_sh;
  kp.lse = a->lse;
  kp.status = a->dev_status;
  kp.num_qtiles = (a->Lq + kBM - 1) / kBM;
  kp.kv_splits = a->kv_splits > 1 ? a->kv_splits : 1;
  kp.part_o = a->part_o;
  kp.part_lse = a->part_lse;
  if (a->scatter != nullptr) {
    const hyb_part_scatter* sc = a->scatter;
    if (sc->o == nullptr || sc->lse == nullptr || sc->ranks < 1 || sc->ranks > 64 || sc->rows <= 0 ||
        sc->slices < 1 || sc->slices > 16 || sc->index0 < 0 || sc->index0 + sc->slices > sc->count)
      return fail(HYB_ERR_INVALID_ARG, "attention: bad partial scatter (ranks %d, rows %d, slices %d, index0 %d, count %d)",
                  sc->ranks, sc->rows, sc->slices, sc->index0, sc->count);
    if (static_cast<long long>(sc->ranks) * sc->rows < a->img_len)
      return fail(HYB_ERR_INVALID_ARG, "attention: %d ranks x %d rows do not own the %d image queries", sc->ranks,
                  sc->rows, a->img_len);
    if (a->acc_o != nullptr) return fail(HYB_ERR_INVALID_ARG, "attention: partial scatter with a ring accumulator");
    kp.sc_o = sc->o;
    kp.sc_lse = sc->lse;
    kp.sc_ranks = sc->ranks;
    kp.sc_rows = sc->rows;
    kp.sc_index0 = sc->index0;
    kp.kv_splits = sc->slices;
    return HYB_OK;
  }
  if (kp.kv_splits > 1 && (a->part_o == nullptr || a->part_lse == nullptr || !al16(a->part_o)))
    return fail(HYB_ERR_INVALID_ARG, "attention: kv_splits > 1 needs 16-byte aligned partial buffers");
  return HYB_OK;
}

int attn_core(const hyb_attn_args* a, cudaStream_t stream, long long kv_pitch = 0) {
  AttnKParams kp;
  int rc = fill_params(a, kp);
  if (rc != HYB_OK || a->Lq == 0) return rc;
  if (device_cc_major() != 10) return fail(HYB_ERR_UNSUPPORTED, "attention: requires an sm_100 GPU");
  const int BH = a->B * a->H;
  CUtensorMap mq, mk, mv;
  if ((rc = make_map(&mq, a->q, BH, a->Lq)) != HYB_OK) return rc;
  if ((rc = make_map(&mk, a->k, BH, a->Lk > 0 ? a->Lk : 1, false, kv_pitch)) != HYB_OK) return rc;
  if ((rc = make_map(&mv, a->v, BH, a->Lk > 0 ? a->Lk : 1, a->v_f16 != 0, kv_pitch)) != HYB_OK) return rc;
  const UnitMap um = plan_units(kp, kp.kv_splits, device_sm_count());
  int rc2 = launch_attn2(mq, mk, mv, kp, um, a->v_f16 != 0, stream);
  if (rc2 != HYB_OK || um.max_k <= 1 || kp.sc_o != nullptr) return rc2;  // owners merge scattered rows
  if (BH > 65535) return fail(HYB_ERR_UNSUPPORTED, "attention: %d (batch, head) pairs in one split launch", BH);
  merge_splits_kernel<<<dim3(static_cast<unsigned>((kp.Lq + kMergeRowsPerBlock - 1) / kMergeRowsPerBlock),
                             static_cast<unsigned>(BH)),
                        256, 0, stream>>>(kp, um);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

}  // namespace
}  // namespace hyb

using namespace hyb;

extern "C" int hyb_attn_fwd(const hyb_attn_args* a, void* stream) {
  if (a == nullptr || a->abi_version != HYB_ABI_VERSION)
    return fail(HYB_ERR_INVALID_ARG, "attention: null args or ABI version mismatch");
  return attn_core(a, static_cast<cudaStream_t>(stream));
}

extern "C" int hyb_attn_work_plan(const hyb_attn_args* a, int32_t sms, int32_t* splits, int32_t n) {
  if (a == nullptr || a->abi_version != HYB_ABI_VERSION)
    return fail(HYB_ERR_INVALID_ARG, "work plan: null args or ABI version mismatch");
  AttnKParams kp;
  const int rc = fill_params(a, kp);
  if (rc != HYB_OK) return rc;
  const UnitMap um = plan_units(kp, kp.kv_splits, sms > 0 ? sms : device_sm_count());
  for (int qp = 0; qp < um.npairs && qp < n; ++qp) {
    const int i = um.npairs - 1 - qp;
    splits[qp] = um.uniform > 0 ? um.uniform : um.prefix[i + 1] - um.prefix[i];
  }
  return um.npairs;
}

extern "C" int hyb_merge_partials(int32_t count, int32_t B, int32_t H, int32_t D, int32_t rows, int32_t txt_rows,
                                  const float* part_o, const float* part_lse, void* out_img, int64_t oi_sb,
                                  int64_t oi_st, int64_t oi_sh, void* out_txt, int64_t ot_sb, int64_t ot_st,
                                  int64_t ot_sh, const uint8_t* text_mask, int64_t text_mask_sb, float* lse,
                                  void* stream) {
  if (D != kHD) return fail(HYB_ERR_UNSUPPORTED, "merge partials: head_dim %d != 128", D);
  if (count < 1 || B < 0 || H < 0 || rows < 0 || txt_rows < 0 || part_o == nullptr || part_lse == nullptr ||
      !al16(part_o))
    return fail(HYB_ERR_INVALID_ARG, "merge partials: bad sizes or buffers");
  if ((rows > 0 && (out_img == nullptr || (reinterpret_cast<uintptr_t>(out_img) & 7u) || (oi_sb % 4) || (oi_st % 4) ||
                    (oi_sh % 4))) ||
      (txt_rows > 0 && (out_txt == nullptr || (reinterpret_cast<uintptr_t>(out_txt) & 7u) || (ot_sb % 4) ||
                        (ot_st % 4) || (ot_sh % 4))))
    return fail(HYB_ERR_INVALID_ARG, "merge partials: outputs must be 8-byte aligned rows");
  const long long total = static_cast<long long>(B) * H * (rows + txt_rows);
  if (total == 0) return HYB_OK;
  MergePartialsParams p;
  p.count = count;
  p.B = B;
  p.H = H;
  p.rows = rows;
  p.txt = txt_rows;
  p.o = part_o;
  p.lse = part_lse;
  p.out_img = static_cast<__nv_bfloat16*>(out_img);
  p.oi_b = oi_sb;
  p.oi_t = oi_st;
  p.oi_h = oi_sh;
  p.out_txt = static_cast<__nv_bfloat16*>(out_txt);
  p.ot_b = ot_sb;
  p.ot_t = ot_st;
  p.ot_h = ot_sh;
  p.text_mask = text_mask;
  p.tm_sb = text_mask_sb;
  p.lse_out = lse;
  if (static_cast<long long>(B) * H > 65535)
    return fail(HYB_ERR_UNSUPPORTED, "merge partials: %lld (batch, head) pairs", static_cast<long long>(B) * H);
  merge_partials_kernel<<<dim3(static_cast<unsigned>((rows + txt_rows + kMergeRowsPerBlock - 1) / kMergeRowsPerBlock),
                               static_cast<unsigned>(B * H)),
                          256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_stage_head_major(int32_t B, int32_t L, int32_t H, int32_t D, const hyb_tensor4* src_k,
                                    const hyb_tensor4* src_v, void* dst_k, void* dst_v, void* stream) {
  if (D != kHD) return fail(HYB_ERR_UNSUPPORTED, "stage: head_dim %d != 128", D);
  if (B <= 0 || H <= 0 || L < 0 || src_k == nullptr || dst_k == nullptr || ((src_v == nullptr) != (dst_v == nullptr)))
    return fail(HYB_ERR_INVALID_ARG, "stage: bad sizes or null tensors");
  if (L == 0) return HYB_OK;
  int rc;
  if ((rc = check_view(*src_k, "stage src_k", true)) != HYB_OK) return rc;
  if (src_v != nullptr && (rc = check_view(*src_v, "stage src_v", true)) != HYB_OK) return rc;
  if (!al16(dst_k) || (dst_v != nullptr && !al16(dst_v)))
    return fail(HYB_ERR_INVALID_ARG, "stage: destinations must be 16-byte aligned");
  StageParams sp{};
  sp.B = B;
  sp.H = H;
  sp.L = L;
  sp.nout = src_v != nullptr ? 2 : 1;
  sp.nseg = 1;
  sp.seg[0][0] = seg_of(*src_k, L, 0);
  if (src_v != nullptr) sp.seg[1][0] = seg_of(*src_v, L, 0);
  sp.out[0] = dst_k;
  sp.out[1] = dst_v;
  return launch_stage(sp, static_cast<cudaStream_t>(stream));
}

extern "C" int hyb_ring_gather_stage(int32_t P, int32_t fmt, int32_t L, int32_t H, int32_t D, int32_t Lmax,
                                     const void* const* blocks, int32_t nchunks, const int32_t* bounds,
                                     const int32_t* owner, const int32_t* row0, void* out_k, void* out_v,
                                     int32_t v_f16, void* stream) {
  if (D != kHD) return fail(HYB_ERR_UNSUPPORTED, "gather stage: head_dim %d != 128", D);
  if (fmt != HYB_FMT_E4M3 && fmt != HYB_FMT_INT8) return fail(HYB_ERR_UNSUPPORTED, "gather stage: format %d", fmt);
  if (P <= 0 || P > 64 || L < 0 || H <= 0 || Lmax <= 0 || nchunks <= 0 || nchunks > kMaxGatherChunks ||
      blocks == nullptr || bounds == nullptr || owner == nullptr || row0 == nullptr || !al16(out_k) || !al16(out_v))
    return fail(HYB_ERR_INVALID_ARG, "gather stage: bad arguments (at most %d chunks)", kMaxGatherChunks);
  GatherParams p;
  p.L = L;
  p.H = H;
  p.Lmax = Lmax;
  p.fmt = fmt;
  p.nchunks = nchunks;
  p.v_f16 = v_f16 != 0;
  for (int r = 0; r < P; ++r) {
    if (blocks[r] == nullptr || (reinterpret_cast<uintptr_t>(blocks[r]) & 15u))
      return fail(HYB_ERR_INVALID_ARG, "gather stage: block %d", r);
    p.blocks[r] = static_cast<const uint8_t*>(blocks[r]);
  }
  if (bounds[0] != 0 || bounds[nchunks] != L) return fail(HYB_ERR_INVALID_ARG, "gather stage: chunks must cover [0, L)");
  for (int c = 0; c < nchunks; ++c) {
    if (bounds[c + 1] < bounds[c] || owner[c] < 0 || owner[c] >= P || row0[c] < 0 ||
        row0[c] + (bounds[c + 1] - bounds[c]) > Lmax)
      return fail(HYB_ERR_INVALID_ARG, "gather stage: chunk %d out of range", c);
    p.owner[c] = owner[c];
    p.row0[c] = row0[c];
  }
  for (int c = 0; c <= nchunks; ++c) p.bounds[c] = bounds[c];
  p.out_k = static_cast<__nv_bfloat16*>(out_k);
  p.out_v = static_cast<__nv_bfloat16*>(out_v);
  if (L == 0) return HYB_OK;
  const long long lanes = static_cast<long long>(H) * L * 8;
  if (lanes >= (1LL << 31)) return fail(HYB_ERR_UNSUPPORTED, "gather stage: %lld rows exceed the 32-bit row index", lanes / 8);
  static int per_sm = 0;
  gather_stage_kernel<<<static_cast<unsigned>(wave_blocks(gather_stage_kernel, &per_sm, lanes)), 256, 0,
                        static_cast<cudaStream_t>(stream)>>>(p);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int hyb_fill_key_bits(int32_t B, int32_t Lk, int32_t kwords, uint32_t* bits, void* stream) {
  if (B <= 0 || Lk < 0 || kwords < 0 || static_cast<long long>(kwords) * 32 < Lk || (bits == nullptr && kwords > 0))
    return fail(HYB_ERR_INVALID_ARG, "key bits: %d words cannot hold %d keys", kwords, Lk);
  if (kwords == 0) return HYB_OK;
  key_bits_kernel<<<grid_for(static_cast<long long>(B) * kwords, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      B, Lk, kwords, bits);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}

extern "C" int64_t hyb_cached_attention_workspace_bytes(int32_t B, int32_t H, int32_t D, int32_t valid_len,
                                                        int32_t img_len, int32_t txt_len, int32_t attend_txt) {
  if (D != kHD || B < 0 || H < 0 || valid_len < 0 || img_len < 0 || txt_len < 0) return -1;
  return layout_for(B, H, valid_len, img_len, img_len, txt_len, attend_txt, device_sm_count()).total;
}

extern "C" int64_t hyb_cached_attention_workspace_bytes_ex(int32_t B, int32_t H, int32_t D, int32_t valid_len,
                                                           int32_t img_len, int32_t txt_len, int32_t attend_txt,
                                                           int32_t staged) {
  if (D != kHD || B < 0 || H < 0 || valid_len < 0 || img_len < 0 || txt_len < 0) return -1;
  return layout_for(B, H, valid_len, img_len, img_len, txt_len, attend_txt, device_sm_count(), staged != 0).total;
}

extern "C" int hyb_decode_rows(int32_t B, int32_t n, int32_t H, int32_t D, const hyb_tensor4* src_k,
                               const hyb_tensor4* src_v, void* dst_k, void* dst_v, int64_t pitch, int64_t row0,
                               void* stream) {
  if (D != kHD) return fail(HYB_ERR_UNSUPPORTED, "decode rows: head_dim %d != 128", D);
  if (B < 0 || n < 0 || H <= 0 || src_k == nullptr || src_v == nullptr || dst_k == nullptr || dst_v == nullptr ||
      !al16(dst_k) || !al16(dst_v) || row0 < 0 || row0 + n > pitch || pitch > INT_MAX)
    return fail(HYB_ERR_INVALID_ARG, "decode rows: bad arguments (rows [%lld, %lld) of pitch %lld)", (long long)row0,
                (long long)(row0 + n), (long long)pitch);
  int rc;
  if ((rc = check_view(*src_k, "decode rows K", true)) != HYB_OK) return rc;
  if ((rc = check_view(*src_v, "decode rows V", true)) != HYB_OK) return rc;
  if ((src_k->fmt != HYB_FMT_E4M3 && src_k->fmt != HYB_FMT_INT8) || src_v->fmt != src_k->fmt)
    return fail(HYB_ERR_UNSUPPORTED, "decode rows: K/V must both be E4M3 or INT8 codes");
  if (B == 0 || n == 0) return HYB_OK;
  StageParams sp{};
  sp.B = B;
  sp.H = H;
  sp.L = n;
  sp.out_pitch = pitch;
  sp.out_t0 = static_cast<int>(row0);
  sp.nout = 2;
  sp.nseg = 1;
  sp.seg[0][0] = seg_of(*src_k, n, 0);
  sp.seg[1][0] = seg_of(*src_v, n, 0);
  sp.out[0] = dst_k;
  sp.out[1] = dst_v;
  sp.out_f16[0] = 0;
  sp.out_f16[1] = 1;
  return launch_stage(sp, static_cast<cudaStream_t>(stream));
}

extern "C" int hyb_cached_attention_workspace_layout(int32_t B, int32_t H, int32_t D, int32_t valid_len,
                                                     int32_t img_len, int32_t txt_len, int32_t attend_txt,
                                                     hyb_workspace_layout* out) {
  if (out == nullptr) return fail(HYB_ERR_INVALID_ARG, "workspace layout: null output");
  if (D != kHD) return fail(HYB_ERR_UNSUPPORTED, "workspace layout: head_dim %d != 128", D);
  if (B < 0 || H < 0 || valid_len < 0 || img_len < 0 || txt_len < 0)
    return fail(HYB_ERR_INVALID_ARG, "workspace layout: negative sizes");
  const WorkspaceLayout w = layout_for(B, H, valid_len, img_len, img_len, txt_len, attend_txt, device_sm_count());
  out->q = w.q;
  out->k = w.k;
  out->v = w.v;
  out->kbits = w.kbits;
  out->qbits = w.qbits;
  out->part_o = w.part_o;
  out->part_lse = w.part_lse;
  out->total = w.total;
  out->Lq = w.Lq;
  out->Lk = w.Lk;
  out->kwords = w.kwords;
  out->qwords = w.qwords;
  out->kv_splits = w.kv_splits;
  out->pad_ = 0;
  return HYB_OK;
}

extern "C" int hyb_cached_attention(const hyb_cached_attn_args* a, void* stream_ptr) {
  if (a == nullptr || a->abi_version != HYB_ABI_VERSION)
    return fail(HYB_ERR_INVALID_ARG, "cached attention: null args or ABI version mismatch");
  if (a->D != kHD) return fail(HYB_ERR_UNSUPPORTED, "cached attention: head_dim %d != 128", a->D);
  if (a->B <= 0 || a->H <= 0 || a->valid_len < 0 || a->img_len < 0 || a->txt_len < 0 || a->group_tokens < 0)
    return fail(HYB_ERR_INVALID_ARG, "cached attention: negative sizes");
  if (a->cache_batch != a->B && a->cache_batch != 1)
    return fail(HYB_ERR_INVALID_ARG, "KV-cache batch mismatch: current=%d, cache=%d", a->B, a->cache_batch);
  if (a->img_k_len < 0 || (a->scatter == nullptr && a->img_k_len > 0 && a->img_k_len != a->img_len))
    return fail(HYB_ERR_INVALID_ARG, "cached attention: img_k_len %d differs from img_len %d without a partial "
                "scatter", a->img_k_len, a->img_len);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const int Lh = a->valid_len, Li = a->img_len, Lt = a->txt_len;
  const int Lik = a->img_k_len > 0 ? a->img_k_len : Li;
  const bool staged = a->staged_k != nullptr;
  const WorkspaceLayout w = layout_for(a->B, a->H, Lh, Li, Lik, Lt, a->attend_txt, device_sm_count(), staged);
  if (a->workspace == nullptr || a->workspace_bytes < w.total || !al16(a->workspace))
    return fail(HYB_ERR_WORKSPACE, "cached attention: workspace %lld bytes < %lld needed",
                (long long)a->workspace_bytes, (long long)w.total);
  if (staged && (a->staged_v == nullptr || !al16(a->staged_k) || !al16(a->staged_v) || a->staged_pitch < w.Lk))
    return fail(HYB_ERR_INVALID_ARG,
                "cached attention: staged history needs K and V buffers, 16-byte aligned, with a pitch of at "
                "least %d rows (got %lld)", w.Lk, (long long)a->staged_pitch);
  int rc;
  if (Lh > 0 && !staged) {
    if ((rc = check_view(a->hist_k, "hist_k", true)) != HYB_OK) return rc;
    if ((rc = check_view(a->hist_v, "hist_v", true)) != HYB_OK) return rc;
    if (a->hist_k.fmt != a->hist_v.fmt) return fail(HYB_ERR_INVALID_ARG, "KV cache K/V dtype mismatch");
  }
  if (Li > 0 && (rc = check_view(a->img_q, "img_q", false)) != HYB_OK) return rc;
  if (Lik > 0) {
    if ((rc = check_view(a->img_k, "img_k", true)) != HYB_OK) return rc;
    if ((rc = check_view(a->img_v, "img_v", true)) != HYB_OK) return rc;
  }
  if (Lt > 0) {
    if ((rc = check_view(a->txt_q, "txt_q", false)) != HYB_OK) return rc;
    if (a->attend_txt) {
      if ((rc = check_view(a->txt_k, "txt_k", false)) != HYB_OK) return rc;
      if ((rc = check_view(a->txt_v, "txt_v", false)) != HYB_OK) return rc;
    }
  }
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  __nv_bfloat16* q_all = reinterpret_cast<__nv_bfloat16*>(ws + w.q);
  __nv_bfloat16* k_all = reinterpret_cast<__nv_bfloat16*>(ws + w.k);
  __nv_bfloat16* v_all = reinterpret_cast<__nv_bfloat16*>(ws + w.v);
  uint32_t* kbits = reinterpret_cast<uint32_t*>(ws + w.kbits);
  uint32_t* qbits = reinterpret_cast<uint32_t*>(ws + w.qbits);

  // key / query visibility bitmaps
  MaskParams mp;
  mp.B = a->B;
  mp.Lh = Lh;
  mp.Li = Li;
  mp.Lik = Lik;
  mp.Lt = Lt;
  mp.Lk = w.Lk;
  mp.kwords = w.kwords;
  mp.Lq = w.Lq;
  mp.qwords = w.qwords;
  mp.attend_txt = a->attend_txt;
  mp.hist_rows = staged ? nullptr : a->hist_rows;
  mp.cache_mask = a->cache_mask;
  mp.cm_sb = a->cache_mask_sb;
  mp.cm_bcast = a->cache_batch == 1 ? 1 : 0;
  mp.text_mask = a->text_mask;
  mp.tm_sb = a->text_mask_sb;
  mp.kbits = kbits;
  mp.qbits = qbits;
  mask_kernel<<<grid_for(static_cast<long long>(a->B) * (w.kwords + w.qwords), 256), 256, 0, stream>>>(mp);
  HYB_CHECK_LAUNCH();

  // K / V composition (history decoded in the same pass); with a staged history only the
  // current keys, into rows [Lh, Lk) of the caller's buffers
  if (w.Lk > (staged ? Lh : 0)) {
    StageParams sp{};
    sp.B = a->B;
    sp.H = a->H;
    sp.L = staged ? w.Lk - Lh : w.Lk;
    sp.out_pitch = staged ? a->staged_pitch : 0;
    sp.out_t0 = staged ? Lh : 0;
    sp.nout = 2;
    sp.nseg = 0;
    const hyb_tensor4* srcs[2][3] = {{&a->hist_k, &a->img_k, &a->txt_k}, {&a->hist_v, &a->img_v, &a->txt_v}};
    const int lens[3] = {staged ? 0 : Lh, Lik, a->attend_txt ? Lt : 0};
    for (int si = 0; si < 3; ++si) {
      if (lens[si] == 0) continue;
      for (int o = 0; o < 2; ++o)
        sp.seg[o][sp.nseg] = seg_of(*srcs[o][si], lens[si], (si == 0 && a->cache_batch == 1) ? 1 : 0,
                                    si == 0 ? a->hist_rows : nullptr);
      ++sp.nseg;
    }
    sp.out[0] = staged ? a->staged_k : k_all;
    sp.out[1] = staged ? a->staged_v : v_all;
    sp.out_f16[0] = 0;
    sp.out_f16[1] = 1;   // V (and so P) in fp16 for P.V
    if ((rc = launch_stage(sp, stream)) != HYB_OK) return rc;
  }
  if (w.Lq > 0) {
    StageParams sp{};
    sp.B = a->B;
    sp.H = a->H;
    sp.L = w.Lq;
    sp.nout = 1;
    sp.nseg = 0;
    if (Li > 0) sp.seg[0][sp.nseg++] = seg_of(a->img_q, Li, 0);
    if (Lt > 0) sp.seg[0][sp.nseg++] = seg_of(a->txt_q, Lt, 0);
    sp.out[0] = q_all;
    sp.out[1] = nullptr;
    sp.out_f16[0] = 0;
    sp.out_f16[1] = 0;
    if ((rc = launch_stage(sp, stream)) != HYB_OK) return rc;
  } else {
    return HYB_OK;
  }

  hyb_attn_args at{};
  at.abi_version = HYB_ABI_VERSION;
  at.B = a->B;
  at.H = a->H;
  at.D = a->D;
  at.Lq = w.Lq;
  at.Lk = w.Lk;
  at.hist_len = Lh;
  at.img_len = Li;
  at.img_k_len = Lik;
  at.group_tokens = a->group_tokens;
  at.softmax_scale = a->softmax_scale;
  at.q_pos0 = a->q_pos0;
  at.k_pos0 = a->k_pos0;
  at.q = q_all;
  at.k = staged ? a->staged_k : k_all;
  at.v = staged ? a->staged_v : v_all;
  at.kbits = kbits;
  at.kwords = w.kwords;
  at.qbits = qbits;
  at.qwords = w.qwords;
  at.out_img = a->out_img;
  at.oi_sb = a->oi_sb;
  at.oi_st = a->oi_st;
  at.oi_sh = a->oi_sh;
  at.oi_seg = a->oi_seg > 0 ? a->oi_seg : (Li > 0 ? Li : 1);
  at.oi_sseg = a->oi_seg > 0 ? a->oi_sseg : 0;
  at.out_txt = a->out_txt;
  at.ot_sb = a->ot_sb;
  at.ot_st = a->ot_st;
  at.ot_sh = a->ot_sh;
  at.lse = a->lse;
  at.dev_status = a->dev_status;
  at.kv_splits = w.kv_splits;
  at.v_f16 = 1;
  at.part_o = reinterpret_cast<float*>(ws + w.part_o);
  at.part_lse = reinterpret_cast<float*>(ws + w.part_lse);
  at.scatter = a->scatter;
  return attn_core(&at, stream, staged ? a->staged_pitch : 0);
}

// =========================================================================================
// Allocation-free variant of hyb_cached_attention.
//
// Some callers cannot allocate device memory at the moment they call attention: a serving
// process whose framework has already reserved (nearly) all of HBM in its own pool for the
// KV cache and activations, a latency-critical decode loop that must not call cudaMalloc
// because it can synchronise the whole device, or a plugin host whose FFI passes tensors but
// no allocator.  For them the staging scratch (head-major Q/K/V, the visibility bitmaps and the
// fp32 partial rows of split query pairs) lives in one fixed device array owned by this library.  The array is static device memory:
// every GPU on which this library's kernels are loaded holds it until the process exits.
// Nothing in it has to start at zero: within one call every byte the attention and merge
// kernels read is first written by that call's mask, staging and attention kernels.
// =========================================================================================
static constexpr long long kNoAllocScratchBytes = 64LL << 20;  // 64 MiB per device
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 128;
std::mutex g_noalloc_mu;
// Device address of g_noalloc_scratch per device, and the unique id of the CUDA context it was
// resolved in: a context that was reset and created again loads the module anew, so the
// address is looked up again there instead of reusing a stale one.
void* g_noalloc_addr[kMaxDevices] = {};
unsigned long long g_noalloc_ctx[kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current CUDA context (0 if it cannot be read).
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
    looked_up = true;
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}
}  // namespace

extern "C" int hyb_cached_attention_noalloc(const hyb_cached_attn_args* a, void* stream) {
  if (a == nullptr || a->abi_version != HYB_ABI_VERSION)
    return fail(HYB_ERR_INVALID_ARG, "cached attention (no-alloc): null args or ABI version mismatch");
  if (a->D != kHD) return fail(HYB_ERR_UNSUPPORTED, "cached attention (no-alloc): head_dim %d != 128", a->D);
  if (a->B <= 0 || a->H <= 0 || a->valid_len < 0 || a->img_len < 0 || a->txt_len < 0 || a->group_tokens < 0)
    return fail(HYB_ERR_INVALID_ARG, "cached attention (no-alloc): negative sizes");
  const int64_t need = hyb_cached_attention_workspace_bytes_ex(a->B, a->H, a->D, a->valid_len, a->img_len,
                                                               a->txt_len, a->attend_txt, a->staged_k != nullptr);
  if (need < 0) return fail(HYB_ERR_INVALID_ARG, "cached attention (no-alloc): unsupported sizes");
  if (need > kNoAllocScratchBytes)
    return fail(HYB_ERR_WORKSPACE,
                "cached attention (no-alloc): these sizes need %lld bytes of staging scratch but the "
                "fixed per-device scratch holds %lld; use hyb_cached_attention with a caller workspace",
                (long long)need, (long long)kNoAllocScratchBytes);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(HYB_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(HYB_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  const unsigned long long ctx = current_context_id();
  void* scratch = nullptr;
  {
    // First call on a device (and in each new context of it), with that device current:
    // resolve the array's device address.
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[dev] == nullptr || ctx == 0 || g_noalloc_ctx[dev] != ctx) {
      void* addr = nullptr;
      e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
      if (e != cudaSuccess)
        return fail(HYB_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
      g_noalloc_addr[dev] = addr;
      g_noalloc_ctx[dev] = ctx;
    }
    scratch = g_noalloc_addr[dev];
  }
  hyb_cached_attn_args local = *a;
  local.workspace = scratch;
  local.workspace_bytes = kNoAllocScratchBytes;
  return hyb_cached_attention(&local, stream);
}
