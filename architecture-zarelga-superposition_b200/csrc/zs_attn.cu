// Causal GQA flash attention forward on the 5th-generation tensor cores.
//
// Replaces flash_attn_varlen_func as GatedAttention uses it
// (modeling/attention.py:131-169): causal, optional causal sliding window
// (window W = current token + W-1 previous), optional packed sequences, and
// the learned per-head key sink of modeling/hca.py:138-144,264-298 (one extra
// always-visible key whose value is zero).  Scale 1/sqrt(head_dim).
//
// One CTA per (256 query rows = two 128-row tiles, head, batch row), 320
// threads:
//   warp 0      TMA: both Q tiles once, then K and V tiles of 128 keys into a
//               ring of single-tile slots (K_j, V_j, K_j+1, ...)
//   warp 1      MMA: per key tile j and query tile t, O_t += P_t V_{j-1}
//               (P from tensor memory) then S_t = Q_t K_j^T; the two query
//               tiles alternate, so one tile's softmax overlaps the other
//               tile's products
//   warps 2..5  softmax of query tile 0, warps 6..9 of query tile 1: one
//               row per thread; read S_t from TMEM, keep the running max
//               (log2 domain) and sum, rescale O_t in TMEM only when the max
//               grows by > 8 (2^8 headroom keeps P and the sums finite), write
//               P_t (bf16 pairs) over S_t's first 64 columns; finally O_t /
//               sum and the log-sum-exp.
// TMEM columns: S_t / P_t at t*128 (128), O_t at 256 + t*hd.
#include "zs_common.cuh"

namespace zs {
namespace attn {

constexpr int BQ = 128;      // query rows per tile (two tiles per CTA in the forward)
constexpr int BKV = 128;     // keys per tile
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

struct FwdArgs {
  int B, S, H, Hkv, hd;
  int window;                 // <= 0: none
  float scale_log2;           // softmax scale * log2(e)
  const int* seg_start;       // nullable [B*S]: first position of the token's packed sequence (-1: padding)
  const void* k_sink;         // nullable [H, hd] (dtype of sink_dtype)
  int sink_dtype;
  __nv_bfloat16* o;           // [B*S, H*hd] rows of ldo elements
  int64_t ldo;
  float* lse;                 // [B, H, S] natural-log log-sum-exp
  const __nv_bfloat16* gate;  // nullable [B*S, H] rows of ldg: O is multiplied by sigmoid(gate)
  int64_t ldg;
};

template <int HD>
struct FwdSmem {
  static constexpr int TILE = 128 * HD * 2;          // one 128-row tile (Q, K or V)
  static constexpr int NSLOT = HD == 128 ? 5 : 8;    // K/V ring slots of one tile each
  static constexpr int OFF_Q = 0;                    // two Q tiles
  static constexpr int OFF_KV = 2 * TILE;
  static constexpr int OFF_BAR = OFF_KV + NSLOT * TILE;
  // q_full, kv_full[NSLOT], kv_empty[NSLOT], s_full[2], p_full[2], o_done[2], done
  static constexpr int NBAR = 1 + 2 * NSLOT + 7;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int TOTAL = OFF_MISC + 16;
  static constexpr int ALLOC = TOTAL + 1024;
};

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed f32x2 arithmetic (two lanes of a 64-bit register pair per instruction).
__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  uint32_t a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(a), "=r"(b) : "l"(v));
  lo = __uint_as_float(a);
  hi = __uint_as_float(b);
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const FwdArgs a) {
  using L = FwdSmem<HD>;
  constexpr int NSLOT = L::NSLOT;
  constexpr int ATOMS = HD / 64;           // 128-byte swizzle atoms across head_dim
  constexpr int ATOM_BYTES = 128 * 128;    // 128 rows x 128 bytes
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_seg_lo[2];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + NSLOT;
  uint64_t* s_full = kv_empty + NSLOT;   // [2]
  uint64_t* p_full = s_full + 2;         // [2]
  uint64_t* o_done = p_full + 2;         // [2]
  uint64_t* done = o_done + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qb = (a.S + 2 * BQ - 1) / (2 * BQ);
  const int qb = n_qb - 1 - (int)blockIdx.x;   // heaviest (latest) query blocks first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.H / a.Hkv);
  const int q0 = qb * 2 * BQ;
  const int64_t row0 = (int64_t)b * a.S;

  // key tile range [lo_t, hi_t] of each query tile (cnt_t = 0: the tile is past the sequence)
  if (threadIdx.x < 2) s_seg_lo[threadIdx.x] = 0x7fffffff;
  __syncthreads();
  if (a.seg_start != nullptr && threadIdx.x < 2 * BQ) {
    const int q = q0 + (int)threadIdx.x;
    if (q < a.S) {
      const int st = __ldg(a.seg_start + row0 + q);
      if (st >= 0) atomicMin(&s_seg_lo[threadIdx.x / BQ], st);
    }
  }
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 2);   // one release per query tile
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(done, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  int lo[2], hi[2], cnt[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qt0 = q0 + t * BQ;
    if (qt0 >= a.S) {
      lo[t] = 0;
      hi[t] = -1;
      cnt[t] = 0;
      continue;
    }
    int kf = a.window > 0 ? max(0, qt0 - (a.window - 1)) : 0;
    if (a.seg_start != nullptr && s_seg_lo[t] != 0x7fffffff) kf = max(kf, s_seg_lo[t]);
    lo[t] = kf / BKV;
    hi[t] = min(qt0 + BQ - 1, a.S - 1) / BKV;
    cnt[t] = hi[t] - lo[t] + 1;
  }
  const int ulo = cnt[0] > 0 ? lo[0] : lo[1];
  const int uhi = cnt[1] > 0 ? max(hi[0], hi[1]) : hi[0];
  constexpr uint32_t IDESC_S = idesc_f16(128, 128, 1, 0, 0);
  constexpr uint32_t IDESC_PV = idesc_f16(128, HD, 1, 0, 1);

  if (warp == 0) {
    if (lane == 0) {
      uint32_t issued = 0, par = 0;
      const int nq = cnt[1] > 0 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, nq * L::TILE);
      for (int t = 0; t < nq; ++t)
#pragma unroll
        for (int at = 0; at < ATOMS; ++at)
          tma_load_2d(smem + L::OFF_Q + t * L::TILE + at * ATOM_BYTES, &tmQ, q_full, h * HD + at * 64,
                      (int)(row0 + q0 + t * BQ));
      int item = 0;
      bool ok = true;
      for (int j = ulo; ok && j <= uhi; ++j) {
        const bool need = (j >= lo[0] && j <= hi[0]) || (j >= lo[1] && j <= hi[1]);
        if (!need) continue;
        const int krow = (int)(row0 + j * BKV);
#pragma unroll
        for (int kv = 0; kv < 2; ++kv, ++item) {
          const int st = item % NSLOT;
          if (!mbar_wait(&kv_empty[st], ((item / NSLOT) & 1) ^ 1, s_abort, ZS_DEVERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + L::OFF_KV + st * L::TILE;
          mbar_arrive_expect_tx(&kv_full[st], L::TILE);
#pragma unroll
          for (int at = 0; at < ATOMS; ++at)
            tma_load_2d(dst + at * ATOM_BYTES, kv == 0 ? &tmK : &tmV, &kv_full[st], hk * HD + at * 64, krow);
          issued |= 1u << st;
          par = (par & ~(1u << st)) | ((uint32_t)((item / NSLOT) & 1) << st);
        }
      }
      mbar_wait(q_full, 0, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
      for (int s = 0; s < NSLOT; ++s)
        if (issued & (1u << s)) mbar_wait(&kv_full[s], (par >> s) & 1, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    bool ok = warp_wait(q_full, 0, s_abort, ZS_DEVERR_TIMEOUT_MMA);
    int u[2] = {0, 0};       // key tiles whose S MMA has been issued, per query tile
    int vit[2] = {0, 0};     // ring item of the V tile the pending PV product reads
    bool issued_any = false;
    // O_t += P_t V for the tile's previous key tile, then release that V slot for this query tile
    auto pv = [&](int t) -> bool {
      if (!warp_wait(&p_full[t], (u[t] - 1) & 1, s_abort, ZS_DEVERR_TIMEOUT_MMA)) return false;
      const int vi = vit[t], vs = vi % NSLOT;
      if (!warp_wait(&kv_full[vs], (vi / NSLOT) & 1, s_abort, ZS_DEVERR_TIMEOUT_MMA)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t va = smem_u32(smem + L::OFF_KV + vs * L::TILE);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          tc_mma_f16_ts(tmem + 256 + t * HD, tmem + t * 128 + kk * 8, smem_desc(va + kk * 2048, ATOM_BYTES, 1024, 2),
                        IDESC_PV, (u[t] > 1 || kk > 0) ? 1u : 0u);
        tc_commit(&kv_empty[vs]);
      }
      __syncwarp();
      return true;
    };
    int item = 0;
    for (int j = ulo; ok && j <= uhi; ++j) {
      const bool in0 = j >= lo[0] && j <= hi[0], in1 = j >= lo[1] && j <= hi[1];
      if (!in0 && !in1) continue;
      const int ik = item, iv = item + 1;
      item += 2;
      const int ks = ik % NSLOT;
      if (!warp_wait(&kv_full[ks], (ik / NSLOT) & 1, s_abort, ZS_DEVERR_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const bool in = t == 0 ? in0 : in1;
        if (!in) {
          // this query tile never reads V_j: its share of the slot's release now
          if (lane == 0) tc_commit(&kv_empty[iv % NSLOT]);
          __syncwarp();
          continue;
        }
        if (u[t] > 0 && !pv(t)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t qa = smem_u32(smem + L::OFF_Q + t * L::TILE);
          const uint32_t ka = smem_u32(smem + L::OFF_KV + ks * L::TILE);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk / 4) * ATOM_BYTES + (kk % 4) * 32;
            tc_mma_f16(tmem + t * 128, smem_desc(qa + off, 16, 1024, 2), smem_desc(ka + off, 16, 1024, 2), IDESC_S,
                       kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[t]);
          issued_any = true;
        }
        __syncwarp();
        ++u[t];
        vit[t] = iv;
      }
      if (!ok) break;
      // K_j: both query tiles' S products read it
      if (lane == 0) {
        tc_commit(&kv_empty[ks]);
        tc_commit(&kv_empty[ks]);
      }
      __syncwarp();
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (ok && u[t] > 0) ok = pv(t);
      if (lane == 0) tc_commit(&o_done[t]);
      __syncwarp();
    }
    if (lane == 0 && issued_any) {
      tc_commit(done);
      mbar_wait(done, 0, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
    }
    __syncwarp();
  } else {
    const int t = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qt0 = q0 + t * BQ;
    const int q = qt0 + r;
    const bool qvalid = q < a.S;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t ts = tmem + lane_base + t * 128;
    const int n = cnt[t];
    int qseg = 0;
    if (a.seg_start != nullptr && qvalid) qseg = __ldg(a.seg_start + row0 + q);
    // running max (log2 domain, relative to which P is formed) and sum
    float m_used = -INFINITY, l = 0.f;
    bool ok = n > 0;
    if (ok && a.k_sink != nullptr) {
      // sink logit from this row of the Q tile in shared memory (swizzled 16-byte chunks)
      ok = warp_wait(q_full, 0, s_abort, ZS_DEVERR_TIMEOUT_EPILOGUE);
      if (ok && qvalid) {
        const uint8_t* qrow = smem + L::OFF_Q + t * L::TILE + r * 128;
        float dot = 0.f;
#pragma unroll
        for (int ch = 0; ch < HD / 8; ++ch) {
          const uint4 v = *reinterpret_cast<const uint4*>(qrow + (ch >> 3) * ATOM_BYTES + (((ch & 7) ^ (r & 7)) * 16));
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[x]));
            const int c = ch * 8 + 2 * x;
            float k0, k1;
            if (a.sink_dtype == ZS_F32) {
              k0 = reinterpret_cast<const float*>(a.k_sink)[h * HD + c];
              k1 = reinterpret_cast<const float*>(a.k_sink)[h * HD + c + 1];
            } else {
              k0 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.k_sink)[h * HD + c]);
              k1 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.k_sink)[h * HD + c + 1]);
            }
            dot = fmaf(f.x, k0, dot);
            dot = fmaf(f.y, k1, dot);
          }
        }
        m_used = dot * a.scale_log2;
        l = 1.f;
      }
    }
    const uint64_t scale2 = pack2(__float_as_uint(a.scale_log2), __float_as_uint(a.scale_log2));
    for (int uu = 0; uu < n && ok; ++uu) {
      const int j = lo[t] + uu;
      if (!warp_wait(&s_full[t], uu & 1, s_abort, ZS_DEVERR_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(ts + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tc_wait_ld();
      const int k0 = j * BKV;
      const bool edge = (k0 + BKV - 1 > qt0) || (qt0 + BQ - 1 >= a.S) || a.seg_start != nullptr ||
                        (a.window > 0 && qt0 + BQ - 1 - k0 >= a.window);
      if (edge) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const int k = k0 + c;
          bool vis = qvalid && k <= q;
          if (a.window > 0) vis = vis && (q - k < a.window);
          if (a.seg_start != nullptr) vis = vis && (k >= qseg) && qseg >= 0;
          if (!vis) sr[c] = __float_as_uint(-INFINITY);
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; c += 8) {
        mx0 = fmax3(mx0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        mx1 = fmax3(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
        mx2 = fmax3(mx2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
        mx3 = fmax3(mx3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * a.scale_log2;
      const float m_new = fmaxf(m_used, mx);
      const bool need = m_new > m_used + 8.0f;
      float f = 1.0f;
      if (need) {
        f = (m_used == -INFINITY) ? 0.f : fast_exp2(m_used - m_new);
        l *= f;
        m_used = m_new;
      }
      // O_t holds every earlier product (this S_t was issued after them)
      if (uu >= 1 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t orow[32];
          tmem_ld_32x32b_x32(tmem + lane_base + 256 + t * HD + c * 32, orow);
          tc_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) orow[x] = __float_as_uint(__uint_as_float(orow[x]) * f);
          tmem_st_32x32b_x32(tmem + lane_base + 256 + t * HD + c * 32, orow);
        }
      }
      // P = exp2(s * scale - m_used) (a row with every key so far masked keeps
      // m_used = -inf and all s = -inf: P = 0)
      const float mu = m_used == -INFINITY ? 0.f : m_used;
      const uint64_t negm = pack2(__float_as_uint(-mu), __float_as_uint(-mu));
      uint64_t acc0 = 0, acc1 = 0;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t pw[32];
#pragma unroll
        for (int x = 0; x < 32; x += 2) {
          const int c = hf * 64 + 2 * x;
          float e0, e1, e2, e3;
          unpack2(ffma2(pack2(sr[c], sr[c + 1]), scale2, negm), e0, e1);
          unpack2(ffma2(pack2(sr[c + 2], sr[c + 3]), scale2, negm), e2, e3);
          e0 = fast_exp2(e0);
          e1 = fast_exp2(e1);
          e2 = fast_exp2(e2);
          e3 = fast_exp2(e3);
          acc0 = fadd2(acc0, pack2(__float_as_uint(e0), __float_as_uint(e1)));
          acc1 = fadd2(acc1, pack2(__float_as_uint(e2), __float_as_uint(e3)));
          __nv_bfloat162 p01 = __floats2bfloat162_rn(e0, e1), p23 = __floats2bfloat162_rn(e2, e3);
          pw[x] = *reinterpret_cast<uint32_t*>(&p01);
          pw[x + 1] = *reinterpret_cast<uint32_t*>(&p23);
        }
        tmem_st_32x32b_x32(ts + hf * 32, pw);
      }
      float a0, a1, a2, a3;
      unpack2(acc0, a0, a1);
      unpack2(acc1, a2, a3);
      l += (a0 + a1) + (a2 + a3);
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (ok && warp_wait(&o_done[t], 0, s_abort, ZS_DEVERR_TIMEOUT_EPILOGUE)) {
      tc_fence_after();
      float inv = l > 0.f ? 1.0f / l : 0.f;
      if (a.gate != nullptr && qvalid) {   // the head's output gate, sigmoid in f32
        const float gl = __bfloat162float(a.gate[(row0 + q) * a.ldg + h]);
        inv *= 1.0f / (1.0f + expf(-gl));
      }
      __nv_bfloat16* orow_g = a.o + (row0 + q) * a.ldo + (int64_t)h * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t orow[32];
        tmem_ld_32x32b_x32(tmem + lane_base + 256 + t * HD + c * 32, orow);
        tc_wait_ld();
        if (qvalid) {
          uint4* dst = reinterpret_cast<uint4*>(orow_g + c * 32);
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            uint32_t w[4];
#pragma unroll
            for (int y = 0; y < 4; ++y) {
              __nv_bfloat162 pp = __floats2bfloat162_rn(__uint_as_float(orow[x * 8 + 2 * y]) * inv,
                                                        __uint_as_float(orow[x * 8 + 2 * y + 1]) * inv);
              w[y] = *reinterpret_cast<uint32_t*>(&pp);
            }
            dst[x] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (qvalid) a.lse[((int64_t)b * a.H + h) * a.S + q] = l > 0.f ? (m_used + log2f(l)) * LN2 : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn
}  // namespace zs

using namespace zs;

static bool attn_ld_ok(const void* p, int64_t ld, int64_t width) {
  return p == nullptr || (ld >= width && ld % 8 == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0);
}

extern "C" int zs_gated_attention_forward(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                          int64_t ldv, void* o, int64_t ldo, float* lse, const void* gate_logits,
                                          int64_t ldg, int B, int S, int H, int Hkv, int hd, int window,
                                          const int* seg_start, const void* k_sink, int sink_dtype,
                                          float softmax_scale, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(q && k && v && o && lse, ZS_ERR_ARG);
  ZS_REQUIRE(B >= 1 && S >= 1 && H >= 1 && Hkv >= 1 && H % Hkv == 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(hd == 64 || hd == 128, ZS_ERR_SHAPE);
  ZS_REQUIRE((int64_t)B * S < ((int64_t)1 << 31), ZS_ERR_SHAPE);
  ZS_REQUIRE(k_sink == nullptr || sink_dtype == ZS_F32 || sink_dtype == ZS_BF16, ZS_ERR_DTYPE);
  ZS_REQUIRE(attn_ld_ok(q, ldq, (int64_t)H * hd) && attn_ld_ok(k, ldk, (int64_t)Hkv * hd) &&
                 attn_ld_ok(v, ldv, (int64_t)Hkv * hd) && attn_ld_ok(o, ldo, (int64_t)H * hd),
             ZS_ERR_ALIGN);
  ZS_REQUIRE(gate_logits == nullptr || ldg >= H, ZS_ERR_SHAPE);
  ZS_BIND(q);
  CUtensorMap tq, tk, tv;
  int rc;
  const uint64_t rows = (uint64_t)B * S;
  if ((rc = make_tmap(&tq, q, ZS_BF16, (uint64_t)H * hd, rows, (uint64_t)ldq * 2, 64, 128)) != ZS_OK) return rc;
  if ((rc = make_tmap(&tk, k, ZS_BF16, (uint64_t)Hkv * hd, rows, (uint64_t)ldk * 2, 64, 128)) != ZS_OK) return rc;
  if ((rc = make_tmap(&tv, v, ZS_BF16, (uint64_t)Hkv * hd, rows, (uint64_t)ldv * 2, 64, 128)) != ZS_OK) return rc;
  attn::FwdArgs a{};
  a.B = B;
  a.S = S;
  a.H = H;
  a.Hkv = Hkv;
  a.hd = hd;
  a.window = window;
  a.scale_log2 = softmax_scale * attn::LOG2E;
  a.seg_start = seg_start;
  a.k_sink = k_sink;
  a.sink_dtype = sink_dtype;
  a.o = reinterpret_cast<__nv_bfloat16*>(o);
  a.ldo = ldo;
  a.lse = lse;
  a.gate = reinterpret_cast<const __nv_bfloat16*>(gate_logits);
  a.ldg = ldg;
  dim3 grid((S + 2 * attn::BQ - 1) / (2 * attn::BQ), H, B);
  if (hd == 128) {
    using L = attn::FwdSmem<128>;
    ZS_CUDA_TRY(cudaFuncSetAttribute(attn::attn_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
    attn::attn_fwd_kernel<128><<<grid, 320, L::ALLOC, stream>>>(tq, tk, tv, a);
  } else {
    using L = attn::FwdSmem<64>;
    ZS_CUDA_TRY(cudaFuncSetAttribute(attn::attn_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC));
    attn::attn_fwd_kernel<64><<<grid, 320, L::ALLOC, stream>>>(tq, tk, tv, a);
  }
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" int zs_attention_forward(const void* q, const void* k, const void* v, void* o, float* lse, int B, int S,
                                    int H, int Hkv, int hd, int window, const int* seg_start, const void* k_sink,
                                    int sink_dtype, float softmax_scale, void* stream) {
  const int64_t qw = (int64_t)H * hd, kw = (int64_t)Hkv * hd;
  return zs_gated_attention_forward(q, qw, k, kw, v, kw, o, qw, lse, nullptr, 0, B, S, H, Hkv, hd, window, seg_start,
                                    k_sink, sink_dtype, softmax_scale, stream);
}

// ------------------------------------------------------------------ backward
//
// Two kernels, no atomics, both on tcgen05 with TMEM accumulators:
//   dq kernel   one CTA per (128-row query tile, head, batch row); loops over
//               64-key tiles: S = Q K^T, dP = dO V^T (three TMEM buffers),
//               dS = P (dP - D) (bf16, back into TMEM), dQ += dS K.
//   dkv kernel  one CTA per (128-key tile, kv head, batch row); loops over the
//               GQA group's query heads and 64-row query tiles:
//               S^T = K Q^T, dP^T = V dO^T, P^T and dS^T to shared memory,
//               dV += P^T dO, dK += dS^T Q; the group's heads accumulate in TMEM.
// P = exp(S * scale - lse) uses the forward's log-sum-exp; D = rowsum(dO * O)
// comes from attn_bwd_prep_kernel.  The sink key (value 0) contributes
// dS_sink = -P_sink * D per query row, returned for the caller to fold into
// dQ and the sink parameter.

namespace zs {
namespace attn {

struct BwdArgs {
  int B, S, H, Hkv, hd;
  int window;
  float scale, scale_log2;
  const int* seg_start;
  const float* lse;     // [B, H, S]
  const float* D;       // [B, H, S]
  const void* k_sink;   // nullable [H, hd]
  int sink_dtype;
  const __nv_bfloat16* q;
  int64_t ldq;          // row strides (elements) of q and of the three gradients
  __nv_bfloat16* dq;    // [B*S, H*hd]
  __nv_bfloat16* dk;    // [B*S, Hkv*hd]
  __nv_bfloat16* dv;
  int64_t lddq, lddk, lddv;
};

__device__ __forceinline__ float sink_at(const BwdArgs& a, int i) {
  return a.sink_dtype == ZS_F32 ? __ldg(reinterpret_cast<const float*>(a.k_sink) + i)
                                : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.k_sink)[i]);
}

// D[b, h, q] = sum_d dO * O over the head's row.  With an output gate (the forward
// stored O_g = sigmoid(z) * O): dout is the gradient of O_g, and per (token, head)
//   D      = sum_d dout * O_g   (= sum_d dO * O for dO = sigmoid(z) * dout)
//   do_raw = bf16(sigmoid(z) * dout)               (the attention core's dO)
//   dz     = D * (1 - sigmoid(z))                  (d loss / d gate logit)
// and the gate_pad columns after the H gate-gradient columns are zeroed.
__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo,
                                     const __nv_bfloat16* __restrict__ dout, int64_t lddo,
                                     const __nv_bfloat16* __restrict__ gate, int64_t ldg,
                                     __nv_bfloat16* __restrict__ do_raw, __nv_bfloat16* __restrict__ dgate,
                                     int64_t lddg, int gate_pad, float* __restrict__ D, int B, int S, int H, int hd) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)B * S * H;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < rows; w += warps) {
    const int64_t tok = w / H;
    const int h = (int)(w - tok * H);
    const __nv_bfloat16* po = o + tok * ldo + (int64_t)h * hd;
    const __nv_bfloat16* pd = dout + tok * lddo + (int64_t)h * hd;
    float acc = 0.f;
    for (int c = lane * 2; c < hd; c += 64) {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(po + c));
      const float2 d = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(pd + c));
      acc = fmaf(a.x, d.x, fmaf(a.y, d.y, acc));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    const int64_t b = tok / S, q = tok - b * S;
    if (lane == 0) D[(b * H + h) * S + q] = acc;
    if (gate != nullptr) {
      const float g = 1.0f / (1.0f + expf(-__bfloat162float(gate[tok * ldg + h])));
      __nv_bfloat16* pr = do_raw + tok * (int64_t)H * hd + (int64_t)h * hd;
      for (int c = lane * 2; c < hd; c += 64) {
        const float2 d = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(pd + c));
        *reinterpret_cast<__nv_bfloat162*>(pr + c) = __floats2bfloat162_rn(g * d.x, g * d.y);
      }
      if (lane == 0) dgate[tok * lddg + h] = __float2bfloat16_rn(acc * (1.0f - g));
      if (h == 0 && lane < gate_pad) dgate[tok * lddg + H + lane] = __float2bfloat16_rn(0.f);
    }
  }
}

template <int HD>
struct DqSmem {
  static constexpr int NKS = 4;                 // K/V ring stages
  static constexpr int QT = 128 * HD * 2;       // Q and dO tiles
  static constexpr int KT = 64 * HD * 2;        // K and V tiles of 64 keys
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = QT;
  static constexpr int OFF_KV = 2 * QT;         // NKS x (K, V)
  static constexpr int OFF_BAR = OFF_KV + NKS * 2 * KT;
  // q_full, kv_full[NKS], kv_empty[NKS], sp_full[3], ds_full[3], done
  static constexpr int NBAR = 1 + 2 * NKS + 6 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int ALLOC = OFF_MISC + 16 + 1024;
};

// dQ per 128-row query tile.  448 threads: warp 0 TMA, warp 1 MMA, warps 2..5,
// 6..9 and 10..13 three softmax groups taking every third 64-key tile, each with
// its own TMEM buffer (S in columns [0, 64), dP in [64, 128) of buffer g at
// g*128; dQ at 384); dS (bf16 pairs) goes back over S's columns, 16 keys at a
// time, and feeds dQ += dS K as the A operand straight from tensor memory.  The
// MMA warp issues S/dP of tile j, then dQ of tile j-2 once its dS is ready:
// three tiles are in flight, so the softmax round trip of one tile overlaps the
// products of the next two (measured: 27 % fewer cycles per tile than with two
// groups).  The sink key (value 0) adds dS_sink = -P_sink * D per row; dQ gains
// dS_sink * k_sink.
template <int HD>
__global__ void __launch_bounds__(448, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmK64, const __grid_constant__ CUtensorMap tmV64,
                       const BwdArgs a, float* __restrict__ ds_sink) {
  using L = DqSmem<HD>;
  constexpr int NKS = L::NKS;
  constexpr int ATOMS = HD / 64;
  constexpr int A128 = 128 * 128, A64 = 64 * 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + NKS;
  uint64_t* sp_full = kv_empty + NKS;   // [3]
  uint64_t* ds_full = sp_full + 3;      // [3]
  uint64_t* done = ds_full + 3;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (a.S + 127) / 128;
  const int qt = n_qt - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.H / a.Hkv);
  const int q0 = qt * 128;
  const int64_t row0 = (int64_t)b * a.S;
  int k_first = a.window > 0 ? max(0, q0 - (a.window - 1)) : 0;
  if (a.seg_start != nullptr) {
    __shared__ int s_lo;
    if (threadIdx.x == 0) s_lo = 0x7fffffff;
    __syncthreads();
    if (threadIdx.x < 128 && q0 + (int)threadIdx.x < a.S) {
      const int st = __ldg(a.seg_start + row0 + q0 + threadIdx.x);
      if (st >= 0) atomicMin(&s_lo, st);
    }
    __syncthreads();
    if (s_lo != 0x7fffffff) k_first = max(k_first, s_lo);
  }
  const int kt_lo = k_first / 64;
  const int kt_hi = min(q0 + 127, a.S - 1) / 64;
  const int n_kv = kt_hi - kt_lo + 1;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NKS; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 3; ++s) {
      mbar_init(&sp_full[s], 1);
      mbar_init(&ds_full[s], 128);
    }
    mbar_init(done, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  // TMEM: buffer g at g*128 (S / dS in [0, 64), dP in [64, 128)), dQ at 384
  constexpr uint32_t IDESC_SP = idesc_f16(128, 64, 1, 0, 0);
  constexpr uint32_t IDESC_DQ = idesc_f16(128, HD, 1, 0, 1);
  if (warp == 0) {
    if (lane == 0) {
      uint32_t issued = 0, par = 0;
      mbar_arrive_expect_tx(q_full, 2 * L::QT);
      for (int at = 0; at < ATOMS; ++at) {
        tma_load_2d(smem + L::OFF_Q + at * A128, &tmQ, q_full, h * HD + at * 64, (int)(row0 + q0));
        tma_load_2d(smem + L::OFF_DO + at * A128, &tmDO, q_full, h * HD + at * 64, (int)(row0 + q0));
      }
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % NKS;
        if (!mbar_wait(&kv_empty[st], ((j / NKS) & 1) ^ 1, s_abort, ZS_DEVERR_TIMEOUT_PRODUCER)) break;
        uint8_t* kb = smem + L::OFF_KV + st * 2 * L::KT;
        mbar_arrive_expect_tx(&kv_full[st], 2 * L::KT);
        const int krow = (int)(row0 + (kt_lo + j) * 64);
        for (int at = 0; at < ATOMS; ++at) {
          tma_load_2d(kb + at * A64, &tmK64, &kv_full[st], hk * HD + at * 64, krow);
          tma_load_2d(kb + L::KT + at * A64, &tmV64, &kv_full[st], hk * HD + at * 64, krow);
        }
        issued |= 1u << st;
        par = (par & ~(1u << st)) | ((uint32_t)((j / NKS) & 1) << st);
      }
      mbar_wait(q_full, 0, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
      for (int s = 0; s < NKS; ++s)
        if (issued & (1u << s)) mbar_wait(&kv_full[s], (par >> s) & 1, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    bool ok = warp_wait(q_full, 0, s_abort, ZS_DEVERR_TIMEOUT_MMA);
    bool any = false;
    for (int j = 0; ok && j <= n_kv + 1; ++j) {
      if (j < n_kv) {
        const int st = j % NKS, g = j % 3;
        if (!warp_wait(&kv_full[st], (j / NKS) & 1, s_abort, ZS_DEVERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t qa = smem_u32(smem + L::OFF_Q), da = smem_u32(smem + L::OFF_DO);
          const uint32_t ka = smem_u32(smem + L::OFF_KV + st * 2 * L::KT), va = ka + L::KT;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t offa = (kk / 4) * A128 + (kk % 4) * 32, offb = (kk / 4) * A64 + (kk % 4) * 32;
            tc_mma_f16(tmem + g * 128, smem_desc(qa + offa, 16, 1024, 2), smem_desc(ka + offb, 16, 1024, 2),
                       IDESC_SP, kk > 0);
            tc_mma_f16(tmem + g * 128 + 64, smem_desc(da + offa, 16, 1024, 2), smem_desc(va + offb, 16, 1024, 2),
                       IDESC_SP, kk > 0);
          }
          tc_commit(&sp_full[g]);
          any = true;
        }
        __syncwarp();
      }
      if (j >= 2 && j - 2 < n_kv) {
        const int jj = j - 2, st = jj % NKS, g = jj % 3;
        if (!warp_wait(&ds_full[g], (jj / 3) & 1, s_abort, ZS_DEVERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t ka = smem_u32(smem + L::OFF_KV + st * 2 * L::KT);
#pragma unroll
          for (int kk = 0; kk < 64 / 16; ++kk)
            tc_mma_f16_ts(tmem + 384, tmem + g * 128 + kk * 8, smem_desc(ka + kk * 2048, A64, 1024, 2), IDESC_DQ,
                          (jj > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&kv_empty[st]);
        }
        __syncwarp();
      }
    }
    if (lane == 0 && any) {
      tc_commit(done);
      mbar_wait(done, 0, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
    }
    __syncwarp();
  } else {
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int q = q0 + r;
    const bool qvalid = q < a.S;
    const uint32_t lb = (uint32_t)(quarter * 32) << 16;
    const uint32_t tb = tmem + lb + grp * 128;
    const int64_t bh = (int64_t)b * a.H + h;
    const float lse2 = qvalid ? __ldg(a.lse + bh * a.S + q) * LOG2E : 0.f;
    const float Dq = qvalid ? __ldg(a.D + bh * a.S + q) : 0.f;
    int qseg = 0;
    if (a.seg_start != nullptr && qvalid) qseg = __ldg(a.seg_start + row0 + q);
    const uint64_t sc2 = pack2(__float_as_uint(a.scale_log2), __float_as_uint(a.scale_log2));
    const uint64_t nl2 = pack2(__float_as_uint(-lse2), __float_as_uint(-lse2));
    const uint64_t nd2 = pack2(__float_as_uint(-Dq), __float_as_uint(-Dq));
    bool ok = true;
    for (int j = grp; j < n_kv && ok; j += 3) {
      const int u = j / 3;
      if (!warp_wait(&sp_full[grp], u & 1, s_abort, ZS_DEVERR_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = (kt_lo + j) * 64;
      const bool edge = (k0 + 63 > q0) || (q0 + 127 >= a.S) || a.seg_start != nullptr ||
                        (a.window > 0 && q0 + 127 - k0 >= a.window);
      // 16 keys at a time; dS (bf16 pairs) overwrites S columns already read
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t sr[16], dr[16];
        tmem_ld_32x32b_x16(tb + ch * 16, sr);
        tmem_ld_32x32b_x16(tb + 64 + ch * 16, dr);
        tc_wait_ld();
        // element pairs in packed f32x2 arithmetic (half the instructions of the scalar
        // form, which issued at about a third of this rate)
        uint32_t w[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          float e0, e1;
          unpack2(ffma2(pack2(sr[2 * x], sr[2 * x + 1]), sc2, nl2), e0, e1);
          float p0 = fast_exp2(e0), p1 = fast_exp2(e1);
          if (edge) {
            const int kk = k0 + ch * 16 + 2 * x;
            bool v0 = qvalid && kk <= q, v1 = qvalid && kk + 1 <= q;
            if (a.window > 0) {
              v0 = v0 && (q - kk < a.window);
              v1 = v1 && (q - kk - 1 < a.window);
            }
            if (a.seg_start != nullptr) {
              v0 = v0 && kk >= qseg && qseg >= 0;
              v1 = v1 && kk + 1 >= qseg && qseg >= 0;
            }
            p0 = v0 ? p0 : 0.f;
            p1 = v1 ? p1 : 0.f;
          } else if (!qvalid) {
            p0 = p1 = 0.f;
          }
          float r0, r1;
          unpack2(fmul2(pack2(__float_as_uint(p0), __float_as_uint(p1)), fadd2(pack2(dr[2 * x], dr[2 * x + 1]), nd2)),
                  r0, r1);
          __nv_bfloat162 pp = __floats2bfloat162_rn(r0, r1);
          w[x] = *reinterpret_cast<uint32_t*>(&pp);
        }
        tmem_st_32x32b_x8(tb + ch * 8, w);
      }
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&ds_full[grp]);
    }
    // all dQ products (the MMA warp's single-phase commit); groups 0 and 1 write
    // dQ columns [g*HD/2, (g+1)*HD/2)
    if (grp < 2 && ok && warp_wait(done, 0, s_abort, ZS_DEVERR_TIMEOUT_EPILOGUE)) {
      tc_fence_after();
      float dss = 0.f;
      if (a.k_sink != nullptr && qvalid) {
        const __nv_bfloat16* qr = a.q + (row0 + q) * a.ldq + (int64_t)h * HD;
        float dot = 0.f;
        for (int c = 0; c < HD; ++c) dot = fmaf(__bfloat162float(qr[c]), sink_at(a, h * HD + c), dot);
        dss = -fast_exp2(dot * a.scale_log2 - lse2) * Dq;
        if (grp == 0) ds_sink[bh * a.S + q] = dss;
      }
      __nv_bfloat16* out = a.dq + (row0 + q) * a.lddq + (int64_t)h * HD;
#pragma unroll 1
      for (int c = grp * (HD / 64); c < (grp + 1) * (HD / 64); ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lb + 384 + c * 32, v);
        tc_wait_ld();
        if (qvalid) {
          uint4* dst = reinterpret_cast<uint4*>(out + c * 32);
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            uint32_t w[4];
#pragma unroll
            for (int y = 0; y < 4; ++y) {
              const int cc = c * 32 + x * 8 + 2 * y;
              float v0 = __uint_as_float(v[x * 8 + 2 * y]), v1 = __uint_as_float(v[x * 8 + 2 * y + 1]);
              if (a.k_sink != nullptr) {
                v0 = fmaf(dss, sink_at(a, h * HD + cc), v0);
                v1 = fmaf(dss, sink_at(a, h * HD + cc + 1), v1);
              }
              __nv_bfloat162 pp = __floats2bfloat162_rn(v0 * a.scale, v1 * a.scale);
              w[y] = *reinterpret_cast<uint32_t*>(&pp);
            }
            dst[x] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int HD>
struct DkvSmem {
  static constexpr int NQS = 4;                     // Q/dO ring stages
  static constexpr int KT = 128 * HD * 2;           // K and V tiles of 128 keys
  static constexpr int QT = 64 * HD * 2;            // Q and dO tiles of 64 rows
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = KT;
  static constexpr int OFF_QD = 2 * KT;             // NQS x (Q, dO)
  static constexpr int OFF_LD = OFF_QD + NQS * 2 * QT;  // [2 groups][2] x (lse2[64], D[64], seg[64])
  static constexpr int OFF_BAR = OFF_LD + 4 * 192 * 4;
  // kv_full, qd_full[NQS], qd_empty[NQS], sp_full[2], ds_full[2], done, ld_full[4]
  static constexpr int NBAR = 1 + 2 * NQS + 4 + 1 + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int ALLOC = OFF_MISC + 16 + 1024;
};

// 320 threads: warp 0 TMA, warp 1 MMA, warps 2..5 and 6..9 two softmax groups
// taking alternate query tiles (group g: iterations i = g, g+2, ...), each with
// its own TMEM buffer: S^T (64 f32 columns) and dP^T (64 columns) come in from
// the MMA, P^T and dS^T (bf16 pairs, 32 columns each) go back into the same
// columns and feed the dV / dK products as the A operand straight from tensor
// memory.  The tensor pipe executes this CTA's MMAs in issue order, so the
// next S^T into a buffer (issued after that buffer's dV/dK) cannot overwrite
// P^T/dS^T before they are read.
template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmQ64, const __grid_constant__ CUtensorMap tmDO64,
                        const BwdArgs a) {
  using L = DkvSmem<HD>;
  constexpr int NQS = L::NQS;
  constexpr int ATOMS = HD / 64;
  constexpr int A128 = 128 * 128, A64 = 64 * 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;
  uint64_t* qd_empty = qd_full + NQS;
  uint64_t* sp_full = qd_empty + NQS;   // [2]
  uint64_t* ds_full = sp_full + 2;      // [2]
  uint64_t* done = ds_full + 2;
  uint64_t* ld_full = done + 1;         // [4]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  float* s_ld = reinterpret_cast<float*>(smem + L::OFF_LD);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int G = a.H / a.Hkv;
  const int k0 = kt * 128;
  const int64_t row0 = (int64_t)b * a.S;
  const int qt_lo = k0 / 64;
  int q_last = a.S - 1;
  if (a.window > 0) q_last = min(q_last, k0 + 127 + a.window - 1);
  const int qt_hi = q_last / 64;
  const int n_q = qt_hi - qt_lo + 1;        // per query head
  const int n_it = G * n_q;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < NQS; ++s) {
      mbar_init(&qd_full[s], 1);
      mbar_init(&qd_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sp_full[s], 1);
      mbar_init(&ds_full[s], 128);
    }
    mbar_init(done, 1);
    for (int s = 0; s < 4; ++s) mbar_init(&ld_full[s], 128);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  // TMEM: buffer g at g*128 (S^T / P^T in columns [0, 64), dP^T / dS^T in [64, 128)),
  // dV at 256, dK at 256 + HD
  constexpr uint32_t IDESC_SP = idesc_f16(128, 64, 1, 0, 0);
  constexpr uint32_t IDESC_ACC = idesc_f16(128, HD, 1, 0, 1);
  if (warp == 0) {
    if (lane == 0 && k0 < a.S) {
      uint32_t issued = 0, par = 0;
      mbar_arrive_expect_tx(kv_full, 2 * L::KT);
      for (int at = 0; at < ATOMS; ++at) {
        tma_load_2d(smem + L::OFF_K + at * A128, &tmK, kv_full, hk * HD + at * 64, (int)(row0 + k0));
        tma_load_2d(smem + L::OFF_V + at * A128, &tmV, kv_full, hk * HD + at * 64, (int)(row0 + k0));
      }
      for (int i = 0; i < n_it; ++i) {
        const int st = i % NQS;
        const int g = i / n_q, qi = qt_lo + i % n_q;
        const int h = hk * G + g;
        if (!mbar_wait(&qd_empty[st], ((i / NQS) & 1) ^ 1, s_abort, ZS_DEVERR_TIMEOUT_PRODUCER)) break;
        uint8_t* qb = smem + L::OFF_QD + st * 2 * L::QT;
        mbar_arrive_expect_tx(&qd_full[st], 2 * L::QT);
        for (int at = 0; at < ATOMS; ++at) {
          tma_load_2d(qb + at * A64, &tmQ64, &qd_full[st], h * HD + at * 64, (int)(row0 + qi * 64));
          tma_load_2d(qb + L::QT + at * A64, &tmDO64, &qd_full[st], h * HD + at * 64, (int)(row0 + qi * 64));
        }
        issued |= 1u << st;
        par = (par & ~(1u << st)) | ((uint32_t)((i / NQS) & 1) << st);
      }
      mbar_wait(kv_full, 0, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
      for (int s = 0; s < NQS; ++s)
        if (issued & (1u << s)) mbar_wait(&qd_full[s], (par >> s) & 1, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    bool ok = k0 < a.S && warp_wait(kv_full, 0, s_abort, ZS_DEVERR_TIMEOUT_MMA);
    bool any = false;
    for (int i = 0; ok && i <= n_it; ++i) {
      if (i < n_it) {
        const int st = i % NQS, g = i & 1;
        if (!warp_wait(&qd_full[st], (i / NQS) & 1, s_abort, ZS_DEVERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t ka = smem_u32(smem + L::OFF_K), va = smem_u32(smem + L::OFF_V);
          const uint32_t qa = smem_u32(smem + L::OFF_QD + st * 2 * L::QT), da = qa + L::QT;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t offa = (kk / 4) * A128 + (kk % 4) * 32, offb = (kk / 4) * A64 + (kk % 4) * 32;
            tc_mma_f16(tmem + g * 128, smem_desc(ka + offa, 16, 1024, 2), smem_desc(qa + offb, 16, 1024, 2),
                       IDESC_SP, kk > 0);
            tc_mma_f16(tmem + g * 128 + 64, smem_desc(va + offa, 16, 1024, 2), smem_desc(da + offb, 16, 1024, 2),
                       IDESC_SP, kk > 0);
          }
          tc_commit(&sp_full[g]);
          any = true;
        }
        __syncwarp();
      }
      if (i >= 1) {
        const int ii = i - 1, st = ii % NQS, g = ii & 1;
        if (!warp_wait(&ds_full[g], (ii >> 1) & 1, s_abort, ZS_DEVERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t qa = smem_u32(smem + L::OFF_QD + st * 2 * L::QT), da = qa + L::QT;
#pragma unroll
          for (int kk = 0; kk < 64 / 16; ++kk) {
            tc_mma_f16_ts(tmem + 256, tmem + g * 128 + kk * 8, smem_desc(da + kk * 2048, A64, 1024, 2), IDESC_ACC,
                          (ii > 0 || kk > 0) ? 1u : 0u);
            tc_mma_f16_ts(tmem + 256 + HD, tmem + g * 128 + 64 + kk * 8, smem_desc(qa + kk * 2048, A64, 1024, 2),
                          IDESC_ACC, (ii > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&qd_empty[st]);
        }
        __syncwarp();
      }
    }
    if (lane == 0 && any) {
      tc_commit(done);
      mbar_wait(done, 0, nullptr, ZS_DEVERR_TIMEOUT_DRAIN);
    }
    __syncwarp();
  } else {
    const int grp = (warp - 2) >> 2;          // softmax group
    const int quarter = warp & 3;             // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;        // key row
    const int k = k0 + r;
    const bool kvalid = k < a.S;
    const int tid = ((warp - 2) & 3) * 32 + lane;
    const uint32_t lb = (uint32_t)(quarter * 32) << 16;
    const uint32_t tb = tmem + lb + grp * 128;
    bool ok = k0 < a.S;
    const uint64_t sc2 = pack2(__float_as_uint(a.scale_log2), __float_as_uint(a.scale_log2));
    for (int i = grp; i < n_it && ok; i += 2) {
      const int u = i >> 1;                   // this group's use count
      const int g = i / n_q, qi = qt_lo + i % n_q;
      const int h = hk * G + g;
      const int qb0 = qi * 64;
      const int64_t bh = (int64_t)b * a.H + h;
      // staging buffer (grp, u & 1) was last read at this group's use u - 2; every
      // thread of the group has passed ld_full of use u - 1 since then
      const int li = grp * 2 + (u & 1);
      float* s_lse2 = s_ld + li * 192;
      float* s_D = s_lse2 + 64;
      int* s_seg = reinterpret_cast<int*>(s_lse2 + 128);
      if (tid < 64) {
        const int qq = qb0 + tid;
        s_lse2[tid] = qq < a.S ? __ldg(a.lse + bh * a.S + qq) * LOG2E : INFINITY;
        if (a.seg_start != nullptr) s_seg[tid] = qq < a.S ? __ldg(a.seg_start + row0 + qq) : -1;
      } else {
        const int qq = qb0 + tid - 64;
        s_D[tid - 64] = qq < a.S ? __ldg(a.D + bh * a.S + qq) : 0.f;
      }
      mbar_arrive(&ld_full[li]);
      if (!warp_wait(&ld_full[li], (u >> 1) & 1, s_abort, ZS_DEVERR_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      if (!warp_wait(&sp_full[grp], u & 1, s_abort, ZS_DEVERR_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // masks only on tiles that straddle the diagonal, the window edge, a
      // packed-sequence start, or the end of the sequence
      const bool edge = (qb0 < k0 + 128) || (qb0 + 63 >= a.S) || a.seg_start != nullptr ||
                        (a.window > 0 && qb0 + 63 - k0 >= a.window);
      // 16 query columns at a time: P^T / dS^T (bf16 pairs) overwrite the S^T / dP^T
      // columns already read (chunk ch writes columns [8ch, 8ch+8), read by chunk ch/2)
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t sr[16], dr[16];
        tmem_ld_32x32b_x16(tb + ch * 16, sr);
        tmem_ld_32x32b_x16(tb + 64 + ch * 16, dr);
        tc_wait_ld();
        // column pairs in packed f32x2 arithmetic; the queries' log-sum-exp and D come
        // from the staging buffer as float2
        uint32_t pw[8], dw[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          const int c = ch * 16 + 2 * x;
          const float2 l2 = *reinterpret_cast<const float2*>(s_lse2 + c);
          const float2 d2 = *reinterpret_cast<const float2*>(s_D + c);
          float e0, e1;
          unpack2(ffma2(pack2(sr[2 * x], sr[2 * x + 1]), sc2, pack2(__float_as_uint(-l2.x), __float_as_uint(-l2.y))),
                  e0, e1);
          float p0 = fast_exp2(e0), p1 = fast_exp2(e1);
          bool v0 = kvalid, v1 = kvalid;
          if (edge) {
            const int q = qb0 + c;
            v0 = v0 && q < a.S && q >= k;
            v1 = v1 && q + 1 < a.S && q + 1 >= k;
            if (a.window > 0) {
              v0 = v0 && (q - k < a.window);
              v1 = v1 && (q + 1 - k < a.window);
            }
            if (a.seg_start != nullptr) {
              v0 = v0 && s_seg[c] >= 0 && s_seg[c] <= k;
              v1 = v1 && s_seg[c + 1] >= 0 && s_seg[c + 1] <= k;
            }
          }
          p0 = v0 ? p0 : 0.f;
          p1 = v1 ? p1 : 0.f;
          const uint64_t p2 = pack2(__float_as_uint(p0), __float_as_uint(p1));
          float r0, r1;
          unpack2(fmul2(p2, fadd2(pack2(dr[2 * x], dr[2 * x + 1]),
                                  pack2(__float_as_uint(-d2.x), __float_as_uint(-d2.y)))), r0, r1);
          __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
          __nv_bfloat162 db = __floats2bfloat162_rn(r0, r1);
          pw[x] = *reinterpret_cast<uint32_t*>(&pb);
          dw[x] = *reinterpret_cast<uint32_t*>(&db);
        }
        tmem_st_32x32b_x8(tb + ch * 8, pw);
        tmem_st_32x32b_x8(tb + 64 + ch * 8, dw);
      }
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&ds_full[grp]);
    }
    // all dV/dK products: the MMA warp's single-phase `done` commit; group 0
    // writes dV, group 1 dK
    if (ok && n_it > 0 && warp_wait(done, 0, s_abort, ZS_DEVERR_TIMEOUT_EPILOGUE)) {
      tc_fence_after();
      const int part = grp;
      const float mul = part == 0 ? 1.0f : a.scale;
      __nv_bfloat16* dst_row = (part == 0 ? a.dv + (row0 + k) * a.lddv : a.dk + (row0 + k) * a.lddk) + (int64_t)hk * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + lb + 256 + part * HD + c * 32, v);
        tc_wait_ld();
        if (kvalid) {
          uint4* dst = reinterpret_cast<uint4*>(dst_row + c * 32);
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            uint32_t w[4];
#pragma unroll
            for (int y = 0; y < 4; ++y) {
              __nv_bfloat162 pp = __floats2bfloat162_rn(__uint_as_float(v[x * 8 + 2 * y]) * mul,
                                                        __uint_as_float(v[x * 8 + 2 * y + 1]) * mul);
              w[y] = *reinterpret_cast<uint32_t*>(&pp);
            }
            dst[x] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn
}  // namespace zs

extern "C" size_t zs_gated_attention_backward_workspace(int B, int S, int H, int hd, int gated) {
  return gated ? (size_t)B * S * H * hd * 2 + 256 : 0;
}

extern "C" int zs_gated_attention_backward(
    const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, const void* o, int64_t ldo,
    const void* dout, int64_t lddo, const float* lse, const void* gate_logits, int64_t ldg, void* dq, int64_t lddq,
    void* dk, int64_t lddk, void* dv, int64_t lddv, void* dgate_logits, int64_t lddg, int gate_pad, float* D, int B,
    int S, int H, int Hkv, int hd, int window, const int* seg_start, const void* k_sink, int sink_dtype,
    float* ds_sink, float softmax_scale, void* workspace, size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(q && k && v && o && dout && lse && dq && dk && dv && D, ZS_ERR_ARG);
  ZS_REQUIRE(B >= 1 && S >= 1 && H >= 1 && Hkv >= 1 && H % Hkv == 0, ZS_ERR_SHAPE);
  ZS_REQUIRE(hd == 64 || hd == 128, ZS_ERR_SHAPE);
  ZS_REQUIRE((k_sink == nullptr) == (ds_sink == nullptr), ZS_ERR_ARG);
  ZS_REQUIRE(k_sink == nullptr || sink_dtype == ZS_F32 || sink_dtype == ZS_BF16, ZS_ERR_DTYPE);
  ZS_REQUIRE((int64_t)B * S < ((int64_t)1 << 31), ZS_ERR_SHAPE);
  const int64_t qw = (int64_t)H * hd, kw = (int64_t)Hkv * hd;
  ZS_REQUIRE(attn_ld_ok(q, ldq, qw) && attn_ld_ok(k, ldk, kw) && attn_ld_ok(v, ldv, kw) && attn_ld_ok(o, ldo, qw) &&
                 attn_ld_ok(dout, lddo, qw) && attn_ld_ok(dq, lddq, qw) && attn_ld_ok(dk, lddk, kw) &&
                 attn_ld_ok(dv, lddv, kw),
             ZS_ERR_ALIGN);
  const bool gated = gate_logits != nullptr;
  ZS_REQUIRE(!gated || (dgate_logits != nullptr && ldg >= H && lddg >= H + gate_pad && gate_pad >= 0 &&
                        gate_pad < 32),
             ZS_ERR_ARG);
  ZS_REQUIRE(!gated || (workspace != nullptr &&
                        workspace_bytes >= zs_gated_attention_backward_workspace(B, S, H, hd, 1)),
             ZS_ERR_WORKSPACE);
  ZS_BIND(q);
  // the attention core's dO: dout itself, or sigmoid(gate) * dout in the workspace
  __nv_bfloat16* do_raw =
      gated ? reinterpret_cast<__nv_bfloat16*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255))
            : nullptr;
  const void* dO = gated ? static_cast<const void*>(do_raw) : dout;
  const int64_t lddO = gated ? qw : lddo;
  int64_t blocks = ((int64_t)B * S * H + 7) / 8;
  if (blocks > 148 * 32) blocks = 148 * 32;
  attn::attn_bwd_prep_kernel<<<(unsigned)blocks, 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(o), ldo, reinterpret_cast<const __nv_bfloat16*>(dout), lddo,
      reinterpret_cast<const __nv_bfloat16*>(gate_logits), ldg, do_raw,
      reinterpret_cast<__nv_bfloat16*>(dgate_logits), lddg, gate_pad, D, B, S, H, hd);
  ZS_CUDA_TRY(cudaGetLastError());
  const uint64_t rows = (uint64_t)B * S;
  CUtensorMap tq128, tdo128, tk64, tv64, tk128, tv128, tq64, tdo64;
  int rc;
  if ((rc = make_tmap(&tq128, q, ZS_BF16, qw, rows, ldq * 2, 64, 128)) != ZS_OK) return rc;
  if ((rc = make_tmap(&tdo128, dO, ZS_BF16, qw, rows, lddO * 2, 64, 128)) != ZS_OK) return rc;
  if ((rc = make_tmap(&tq64, q, ZS_BF16, qw, rows, ldq * 2, 64, 64)) != ZS_OK) return rc;
  if ((rc = make_tmap(&tdo64, dO, ZS_BF16, qw, rows, lddO * 2, 64, 64)) != ZS_OK) return rc;
  if ((rc = make_tmap(&tk128, k, ZS_BF16, kw, rows, ldk * 2, 64, 128)) != ZS_OK) return rc;
  if ((rc = make_tmap(&tv128, v, ZS_BF16, kw, rows, ldv * 2, 64, 128)) != ZS_OK) return rc;
  if ((rc = make_tmap(&tk64, k, ZS_BF16, kw, rows, ldk * 2, 64, 64)) != ZS_OK) return rc;
  if ((rc = make_tmap(&tv64, v, ZS_BF16, kw, rows, ldv * 2, 64, 64)) != ZS_OK) return rc;
  attn::BwdArgs a{};
  a.B = B;
  a.S = S;
  a.H = H;
  a.Hkv = Hkv;
  a.hd = hd;
  a.window = window;
  a.scale = softmax_scale;
  a.scale_log2 = softmax_scale * attn::LOG2E;
  a.seg_start = seg_start;
  a.lse = lse;
  a.D = D;
  a.k_sink = k_sink;
  a.sink_dtype = sink_dtype;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.ldq = ldq;
  a.dq = reinterpret_cast<__nv_bfloat16*>(dq);
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  a.lddq = lddq;
  a.lddk = lddk;
  a.lddv = lddv;
  dim3 gq((S + 127) / 128, H, B), gkv((S + 127) / 128, Hkv, B);
  if (hd == 128) {
    ZS_CUDA_TRY(cudaFuncSetAttribute(attn::attn_bwd_dq_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     attn::DqSmem<128>::ALLOC));
    ZS_CUDA_TRY(cudaFuncSetAttribute(attn::attn_bwd_dkv_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     attn::DkvSmem<128>::ALLOC));
    attn::attn_bwd_dq_kernel<128><<<gq, 448, attn::DqSmem<128>::ALLOC, stream>>>(tq128, tdo128, tk64, tv64, a,
                                                                                 ds_sink);
    ZS_CUDA_TRY(cudaGetLastError());
    attn::attn_bwd_dkv_kernel<128><<<gkv, 320, attn::DkvSmem<128>::ALLOC, stream>>>(tk128, tv128, tq64, tdo64, a);
  } else {
    ZS_CUDA_TRY(cudaFuncSetAttribute(attn::attn_bwd_dq_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     attn::DqSmem<64>::ALLOC));
    ZS_CUDA_TRY(cudaFuncSetAttribute(attn::attn_bwd_dkv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     attn::DkvSmem<64>::ALLOC));
    attn::attn_bwd_dq_kernel<64><<<gq, 448, attn::DqSmem<64>::ALLOC, stream>>>(tq128, tdo128, tk64, tv64, a,
                                                                               ds_sink);
    ZS_CUDA_TRY(cudaGetLastError());
    attn::attn_bwd_dkv_kernel<64><<<gkv, 320, attn::DkvSmem<64>::ALLOC, stream>>>(tk128, tv128, tq64, tdo64, a);
  }
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}

extern "C" int zs_attention_backward(const void* q, const void* k, const void* v, const void* o, const void* dout,
                                     const float* lse, void* dq, void* dk, void* dv, float* D, int B, int S, int H,
                                     int Hkv, int hd, int window, const int* seg_start, const void* k_sink,
                                     int sink_dtype, float* ds_sink, float softmax_scale, void* stream) {
  const int64_t qw = (int64_t)H * hd, kw = (int64_t)Hkv * hd;
  return zs_gated_attention_backward(q, qw, k, kw, v, kw, o, qw, dout, qw, lse, nullptr, 0, dq, qw, dk, kw, dv, kw,
                                     nullptr, 0, 0, D, B, S, H, Hkv, hd, window, seg_start, k_sink, sink_dtype,
                                     ds_sink, softmax_scale, nullptr, 0, stream);
}

// ------------------------------------------------------------ sink gradient
// dk_sink[h, :] = scale * sum over rows r = b*S + s of ds_sink[b, h, s] * q[r, h, :]
// in two fixed-order passes (per-chunk partials, then their sum): the same
// result on every run.  One block of 256 threads per (head, chunk of
// SINK_CHUNK rows): four row groups of 64 threads, each thread two columns.
namespace zs {
namespace attn {
constexpr int SINK_CHUNK = 256;

__global__ void __launch_bounds__(256) sink_grad_partial_kernel(const float* __restrict__ ds, const __nv_bfloat16* q,
                                                                int64_t ldq, int S, int H, int hd, int64_t rows,
                                                                int n_chunks, float* __restrict__ part) {
  const int h = blockIdx.y, chunk = blockIdx.x;
  const int g = threadIdx.x >> 6, c2 = (threadIdx.x & 63) * 2;
  __shared__ float red[4][256];
  float a0 = 0.f, a1 = 0.f;
  if (c2 < hd) {
    const int64_t r0 = (int64_t)chunk * SINK_CHUNK;
    const int64_t r1 = min(r0 + SINK_CHUNK, rows);
    for (int64_t r = r0 + g; r < r1; r += 4) {
      const int64_t b = r / S, s = r - b * S;
      const float w = __ldg(ds + (b * H + h) * (int64_t)S + s);
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(q + r * ldq + (int64_t)h * hd + c2);
      const float2 f = __bfloat1622float2(v);
      a0 = fmaf(w, f.x, a0);
      a1 = fmaf(w, f.y, a1);
    }
  }
  red[g][c2] = a0;
  red[g][c2 + 1] = a1;
  __syncthreads();
  if (g == 0 && c2 < hd) {
    float* o = part + ((int64_t)h * n_chunks + chunk) * hd;
    o[c2] = (red[0][c2] + red[1][c2]) + (red[2][c2] + red[3][c2]);
    o[c2 + 1] = (red[0][c2 + 1] + red[1][c2 + 1]) + (red[2][c2 + 1] + red[3][c2 + 1]);
  }
}

__global__ void sink_grad_finish_kernel(const float* __restrict__ part, int n_chunks, int hd, float scale,
                                        float* __restrict__ dk_sink) {
  const int h = blockIdx.x, c = threadIdx.x;
  if (c >= hd) return;
  const float* p = part + (int64_t)h * n_chunks * hd + c;
  float acc = 0.f;
  for (int i = 0; i < n_chunks; ++i) acc += p[(int64_t)i * hd];
  dk_sink[h * hd + c] = acc * scale;
}
}  // namespace attn
}  // namespace zs

extern "C" size_t zs_attention_sink_grad_workspace(int B, int S, int H, int hd) {
  const int64_t rows = (int64_t)B * S;
  const int64_t n_chunks = (rows + attn::SINK_CHUNK - 1) / attn::SINK_CHUNK;
  return (size_t)(H * n_chunks * hd) * sizeof(float) + 256;
}

extern "C" int zs_attention_sink_grad(const float* ds_sink, const void* q, int64_t ldq, int B, int S, int H, int hd,
                                      float softmax_scale, float* dk_sink, void* workspace, size_t workspace_bytes,
                                      void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ZS_REQUIRE(ds_sink && q && dk_sink, ZS_ERR_ARG);
  ZS_REQUIRE(B >= 1 && S >= 1 && H >= 1 && (hd == 64 || hd == 128), ZS_ERR_SHAPE);
  ZS_REQUIRE(ldq >= (int64_t)H * hd && ldq % 2 == 0 && (reinterpret_cast<uintptr_t>(q) & 3) == 0, ZS_ERR_ALIGN);
  ZS_REQUIRE(workspace && workspace_bytes >= zs_attention_sink_grad_workspace(B, S, H, hd), ZS_ERR_WORKSPACE);
  ZS_BIND(q);
  const int64_t rows = (int64_t)B * S;
  const int n_chunks = (int)((rows + attn::SINK_CHUNK - 1) / attn::SINK_CHUNK);
  float* part = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  attn::sink_grad_partial_kernel<<<dim3((unsigned)n_chunks, (unsigned)H), 256, 0, stream>>>(
      ds_sink, reinterpret_cast<const __nv_bfloat16*>(q), ldq, S, H, hd, rows, n_chunks, part);
  ZS_CUDA_TRY(cudaGetLastError());
  attn::sink_grad_finish_kernel<<<(unsigned)H, 128, 0, stream>>>(part, n_chunks, hd, softmax_scale, dk_sink);
  ZS_CUDA_TRY(cudaGetLastError());
  return ZS_OK;
}
