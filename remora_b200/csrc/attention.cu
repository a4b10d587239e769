// attention.cu -- fused softmax attention, O = softmax(Q K^T * scale [+ causal
// mask]) V, on sm_100a tensor cores with fp32 softmax statistics.
//
// The reference has no attention program (README.md:12 lists FlashAttention
// as in progress); the op is softmax attention, scale 1/sqrt(128), causal
// or not, over Q, K, V bf16 [B, H, S, 128] (B=4, H=32, S=4096 at full size).
//
// Persistent: one CTA per SM (320 threads, TMEM allocated once) walks the
// work items (batch*head, 256 query rows), heaviest first under causal
// masking; barrier phases run on across items, and the next item's Q load and
// first S = Q K^T MMAs overlap the current item's output normalisation (O of a
// query tile is overwritten only after its 4 warps have read it: o_empty).
// Roles:
//   warp 0      TMA producer: an item's Q tiles; K and V tiles of 128 rows into a
//               two-stage ring (128-byte swizzle, two 64-column boxes each).
//   warp 1      TMEM owner + MMA issuer.  Two query tiles (softmax groups
//               WG0, WG1) ping-pong: while one group runs its softmax, the
//               tensor core computes the other group's S = Q K^T and P V.
//   warps 2..5  WG0, warps 6..9 WG1: one query row per thread.  S is read
//               from TMEM with tcgen05.ld (no shuffles: a row lives in one
//               thread), online softmax in the exp2 domain, P rounded to
//               bf16 and written back into TMEM over S with tcgen05.st, and
//               consumed from TMEM as the A operand of the P V MMA.
// TMEM: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512) fp32 columns.
// The running max is only raised when it grows by more than 2^8 (the O
// rescale in TMEM is then rare); P is bounded by 2^8 in between, exact
// enough in bf16 and fp32.  Tiles entirely above the causal diagonal are
// never loaded or computed.  (A CTA per item, 2048 CTAs at [4,32,4096,128],
// measured 1.1 % slower causal and 3.5 % slower non-causal, outputs
// bit-identical.)
#include <algorithm>

#include "runtime.cuh"

namespace rb {
namespace attn {

constexpr int BQ = 128, BKV = 128, HD = 128;
constexpr int kThreads = 320;
constexpr uint32_t kTileBytes = 128 * HD * 2;  // 32 KB: one [128, 128] bf16 tile
constexpr uint32_t kHalf = kTileBytes / 2;     // one 64-column box
constexpr uint32_t kQ0 = 0, kQ1 = kTileBytes, kK = 2 * kTileBytes, kV = 4 * kTileBytes;
constexpr uint32_t kBarOffset = 6 * kTileBytes;
constexpr uint32_t kSmemBytes = kBarOffset + 256 + 1024;

struct Params {
  int S, BH;
  int nkv_total;   // ceil(S / 128)
  int nq_chunks;   // ceil(S / 256)
  int causal;
  float sl2;       // scale * log2(e)
  uint16_t* out;   // [BH, S, 128] bf16
};

struct Smem {
  uint64_t q_full;
  uint64_t k_full[2], v_full[2], kv_empty[2];
  uint64_t s_full[2], p_half[2], p_full[2];  // P columns 0-63 stored (and O rescaled) / all
  uint64_t o_final;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ int n_tiles(const Params& p, int q0) {
  if (!p.causal) return p.nkv_total;
  int n = q0 / BKV + 1;
  return n < p.nkv_total ? n : p.nkv_total;
}

}  // namespace attn
}  // namespace rb

namespace rb {
namespace attnp {
using attn::BQ;
using attn::BKV;
using attn::HD;
using attn::kTileBytes;
using attn::kHalf;
using attn::kQ0;
using attn::kK;
using attn::kV;
using attn::kBarOffset;
using attn::kSmemBytes;
constexpr int kThreads = 320;

struct Smem {
  uint64_t q_full, q_empty;
  uint64_t k_full[2], v_full[2], kv_empty[2];
  uint64_t s_full[2], p_half[2], p_full[2];
  uint64_t o_final, o_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

// Work item i (heaviest first under causal masking): (query chunk, batch*head).
__device__ __forceinline__ void item_coords(const attn::Params& p, int i, int& qc, int& bh) {
  const int chunk = p.causal ? p.nq_chunks - 1 - i / p.BH : i / p.BH;
  bh = i % p.BH;
  qc = chunk * 2 * BQ;
}

// Persistent form: one CTA per SM walks the work items; barrier phases run on
// across items, TMEM is allocated once, the next item's Q load and first S
// MMAs overlap the current item's output normalisation.
__global__ void __launch_bounds__(kThreads, 1)
    k_attention_persist(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, attn::Params p, int n_items) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  Smem* sm = reinterpret_cast<Smem*>(smem + kBarOffset);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&sm->q_full, 1);
    mbar_init(&sm->q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm->k_full[i], 1);
      mbar_init(&sm->v_full[i], 1);
      mbar_init(&sm->kv_empty[i], 1);
      mbar_init(&sm->s_full[i], 1);
      mbar_init(&sm->p_half[i], 4);
      mbar_init(&sm->p_full[i], 4);
      mbar_init(&sm->o_empty[i], 4);
    }
    mbar_init(&sm->o_final, 1);
    sm->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm->tmem_base;
  volatile int* abort_flag = &sm->abort_flag;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int g = 0;  // K/V tiles loaded so far (ring position)
      int it = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++it) {
        int qc, bh;
        item_coords(p, item, qc, bh);
        const int n1 = attn::n_tiles(p, qc + BQ);
        if (it > 0 && !mbar_wait(&sm->q_empty, (it - 1) & 1)) { ok = false; break; }
        mbar_arrive_expect_tx(&sm->q_full, 2 * kTileBytes);
        for (int w = 0; w < 2; ++w)
          for (int h = 0; h < 2; ++h)
            tma_load_3d(smem + kQ0 + w * kTileBytes + h * kHalf, &tmQ, &sm->q_full, h * 64,
                        qc + w * BQ, bh);
        for (int j = 0; j < n1; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          if (!mbar_wait(&sm->kv_empty[st], ph ^ 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&sm->k_full[st], kTileBytes);
          for (int h = 0; h < 2; ++h)
            tma_load_3d(smem + kK + st * kTileBytes + h * kHalf, &tmK, &sm->k_full[st], h * 64,
                        j * BKV, bh);
          mbar_arrive_expect_tx(&sm->v_full[st], kTileBytes);
          for (int h = 0; h < 2; ++h)
            tma_load_3d(smem + kV + st * kTileBytes + h * kHalf, &tmV, &sm->v_full[st], h * 64,
                        j * BKV, bh);
        }
      }
      if (!ok) *abort_flag = 1;
      // let the last copies land before the CTA can exit
      if (g > 0) {
        mbar_wait(&sm->k_full[(g - 1) & 1], ((g - 1) >> 1) & 1);
        mbar_wait(&sm->v_full[(g - 1) & 1], ((g - 1) >> 1) & 1);
      }
      if (it > 0) mbar_wait(&sm->q_full, (it - 1) & 1);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t id_s = idesc_bf16_f32(BQ, BKV, 0, 0);
      constexpr uint32_t id_pv = idesc_bf16_f32(BQ, HD, 0, 1);
      const uint32_t sq0 = smem_u32(smem + kQ0);
      const uint32_t sk = smem_u32(smem + kK), sv = smem_u32(smem + kV);
      int g = 0;            // K/V tiles consumed (ring position)
      int gw[2] = {0, 0};   // key tiles of each query tile so far (s/p barrier parity)
      int it = 0;
      bool ok = true;
      auto issue_s = [&](int w, int st) {
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
          mma_bf16_ss(tbase + w * BKV, smem_desc_sw128(sq0 + w * kTileBytes + off, 16, 1024),
                      smem_desc_sw128(sk + st * kTileBytes + off, 16, 1024), id_s, k > 0);
        }
        mma_commit(&sm->s_full[w]);
      };
      auto issue_pv = [&](int w, int st, bool first, int k0) {
#pragma unroll
        for (int k = k0; k < k0 + BKV / 32; ++k)
          mma_bf16_ts(tbase + 256 + w * HD, tbase + w * BKV + k * 8,
                      smem_desc_sw128(sv + st * kTileBytes + k * 2048, kHalf, 1024), id_pv,
                      (!first || k > 0) ? 1u : 0u);
      };
      // P.V of query tile w's key tile j (its gw-th overall)
      auto pv = [&](int w, int st, int j) -> bool {
        const int gp = gw[w];
        if (j == 0 && it > 0) {  // O_w still holds the last item's output until read
          if (!mbar_wait(&sm->o_empty[w], (it - 1) & 1)) return false;
        }
        if (!mbar_wait(&sm->p_half[w], gp & 1)) return false;
        tc_fence_after();
        issue_pv(w, st, j == 0, 0);
        if (!mbar_wait(&sm->p_full[w], gp & 1)) return false;
        tc_fence_after();
        issue_pv(w, st, j == 0, BKV / 32);
        ++gw[w];
        return true;
      };
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++it) {
        int qc, bh;
        item_coords(p, item, qc, bh);
        const int n0 = attn::n_tiles(p, qc), n1 = attn::n_tiles(p, qc + BQ);
        ok = mbar_wait(&sm->q_full, it & 1) && mbar_wait(&sm->k_full[g & 1], (g >> 1) & 1);
        if (!ok) break;
        tc_fence_after();
        issue_s(0, g & 1);
        issue_s(1, g & 1);
        if (n1 == 1) mma_commit(&sm->q_empty);
        for (int j = 0; ok && j < n1; ++j, ++g) {
          const int st = g & 1, stn = (g + 1) & 1;
          const uint32_t phn = ((g + 1) >> 1) & 1;
          if (!mbar_wait(&sm->v_full[st], (g >> 1) & 1)) { ok = false; break; }
          if (j < n0) {
            if (!pv(0, st, j)) { ok = false; break; }
            if (j + 1 < n0) {
              if (!mbar_wait(&sm->k_full[stn], phn)) { ok = false; break; }
              tc_fence_after();
              issue_s(0, stn);
            }
          }
          if (!pv(1, st, j)) { ok = false; break; }
          mma_commit(&sm->kv_empty[st]);
          if (j + 1 < n1) {
            if (!mbar_wait(&sm->k_full[stn], phn)) { ok = false; break; }
            tc_fence_after();
            issue_s(1, stn);
            if (j + 2 == n1) mma_commit(&sm->q_empty);  // the item's last S read Q
          }
        }
        mma_commit(&sm->o_final);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    const int w = (warp - 2) >> 2;
    const int lg = warp & 3;
    const int row = lg * 32 + lane;
    const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
    const uint32_t t_s = tbase + lane_off + w * BKV;
    const uint32_t t_o = tbase + lane_off + 256 + w * HD;
    int gs = 0;  // key tiles of this query tile so far (s/p barrier parity)
    int it = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++it) {
      int qc, bh;
      item_coords(p, item, qc, bh);
      const int q0w = qc + w * BQ;
      const int q_row = q0w + row;
      const int n_w = attn::n_tiles(p, q0w);
      float m = -INFINITY, l = 0.0f;
      for (int j = 0; j < n_w; ++j, ++gs) {
        bool got = !*abort_flag && mbar_wait(&sm->s_full[w], gs & 1);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        tc_fence_after();
        uint32_t r[128];
        tmem_ld32(t_s + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld32(t_s + 64, *reinterpret_cast<uint32_t(*)[32]>(&r[64]));
        tmem_ld32(t_s + 96, *reinterpret_cast<uint32_t(*)[32]>(&r[96]));
        tmem_ld_wait();
        const int kv0 = j * BKV;
        const bool mask = (p.causal && kv0 + BKV - 1 > q0w) || kv0 + BKV > p.S;
        if (mask) {
          const int lim = p.causal ? min(q_row + 1, p.S) : p.S;
#pragma unroll
          for (int c = 0; c < BKV; ++c)
            r[c] = (kv0 + c >= lim) ? 0xff800000u : r[c];
        }
        float pm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = __uint_as_float(r[i]);
#pragma unroll
        for (int c = 8; c < BKV; ++c) pm[c & 7] = fmaxf(pm[c & 7], __uint_as_float(r[c]));
        const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                               fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
        const float mt = mx * p.sl2;
        const bool raise = mt > m + 8.0f;
        const float alpha = raise ? ((m == -INFINITY) ? 0.0f : attn::ex2(m - mt)) : 1.0f;
        const bool rescale_o = raise && j > 0 && m != -INFINITY;
        if (raise) {
          l *= alpha;
          m = mt;
        }
        const float mu = (m == -INFINITY) ? 0.0f : m;
        float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < BKV / 2; c += 2) {
          const float a = attn::ex2(fmaf(__uint_as_float(r[c]), p.sl2, -mu));
          const float b = attn::ex2(fmaf(__uint_as_float(r[c + 1]), p.sl2, -mu));
          ps[(c >> 1) & 7] += a + b;
          r[c >> 1] = pack_bf16x2(a, b);
        }
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tmem_st16(t_s + c * 16, *reinterpret_cast<const uint32_t(*)[16]>(&r[c * 16]));
        if (__any_sync(0xffffffffu, rescale_o)) {
          const float f = rescale_o ? alpha : 1.0f;
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            uint32_t o[32];
            tmem_ld32(t_o + c, o);
            tmem_ld_wait();
            uint32_t lo[16], hi[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              lo[i] = __float_as_uint(__uint_as_float(o[i]) * f);
              hi[i] = __float_as_uint(__uint_as_float(o[16 + i]) * f);
            }
            tmem_st16(t_o + c, lo);
            tmem_st16(t_o + c + 16, hi);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm->p_half[w]);
#pragma unroll
        for (int c = BKV / 2; c < BKV; c += 2) {
          const float a = attn::ex2(fmaf(__uint_as_float(r[c]), p.sl2, -mu));
          const float b = attn::ex2(fmaf(__uint_as_float(r[c + 1]), p.sl2, -mu));
          ps[(c >> 1) & 7] += a + b;
          r[c >> 1] = pack_bf16x2(a, b);
        }
        l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
#pragma unroll
        for (int c = 2; c < 4; ++c)
          tmem_st16(t_s + c * 16, *reinterpret_cast<const uint32_t(*)[16]>(&r[c * 16]));
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm->p_full[w]);
      }
      if (!ok) break;
      bool fin = !*abort_flag && mbar_wait(&sm->o_final, it & 1) && !*abort_flag;
      if (!__all_sync(0xffffffffu, fin)) { ok = false; break; }
      tc_fence_after();
      const float inv = 1.0f / l;
      uint16_t* dst = p.out + ((int64_t)bh * p.S + q_row) * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t o[32];
        tmem_ld32(t_o + c, o);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        if (q_row < p.S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm->o_empty[w]);  // O_w read: the next item may overwrite it
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}
}  // namespace attnp
}  // namespace rb


extern "C" int remora_b200_attention_fwd_bf16(const void* q, const void* k, const void* v,
                                              void* out, int64_t batch, int64_t heads,
                                              int64_t seq, int64_t head_dim, int causal,
                                              float scale, void* stream) {
  using namespace rb;
  using namespace rb::attn;
  clear_error();
  RB_CHECK_ARG(batch >= 0 && heads >= 0 && seq >= 0, "attention: bad sizes");
  RB_CHECK_ARG(head_dim == HD, "attention: head_dim %lld unsupported (128 only)",
               (long long)head_dim);
  const int64_t BH = batch * heads;
  if (BH == 0 || seq == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(q && k && v && out, "attention: null pointer");
  RB_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out),
               "attention: q, k, v and out must be 16-byte aligned");
  RB_CHECK_ARG(seq < (1 << 30) && BH < (1 << 30), "attention: sizes exceed 2^30");
  RB_CHECK_ARG(scale > 0.0f && scale == scale, "attention: scale must be positive");
  CUtensorMap tq, tk, tv;
  uint64_t d[3] = {(uint64_t)HD, (uint64_t)seq, (uint64_t)BH};
  uint64_t s[2] = {(uint64_t)HD * 2, (uint64_t)seq * HD * 2};
  uint32_t box[3] = {64, 128, 1};
  int rc;
  if ((rc = make_tmap(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, s, box,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, s, box,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, s, box,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  Params p;
  p.S = (int)seq;
  p.BH = (int)BH;
  p.nkv_total = (int)((seq + BKV - 1) / BKV);
  p.nq_chunks = (int)((seq + 2 * BQ - 1) / (2 * BQ));
  p.causal = causal ? 1 : 0;
  p.sl2 = scale * 1.4426950408889634f;
  p.out = static_cast<uint16_t*>(out);
  const int64_t grid = (int64_t)p.nq_chunks * BH;
  RB_CHECK_ARG(grid < (1ll << 31), "attention: grid too large");
  const int n_items = (int)grid;
  const int ctas = std::min(n_items, num_sms());
  RB_CUDA(cudaFuncSetAttribute(attnp::k_attention_persist,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
  attnp::k_attention_persist<<<(unsigned)ctas, attnp::kThreads, kSmemBytes, as_stream(stream)>>>(
      tq, tk, tv, p, n_items);
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}
