// Scaled dot-product attention forward (flash-style, causal or not) on sm_100a.
//
// One CTA = 128 query rows of one (batch, head); 4 warps, one query row per
// thread.  Per key block of 128: thread 0 issues S = Q K^T (tcgen05.mma,
// kind::tf32 for f32 inputs, kind::f16 for bf16) into TMEM; every thread reads
// its row of S (tcgen05.ld), applies scale and the causal mask, updates the
// running max / sum in f32 and writes P to shared memory in the UMMA operand
// layout (128-byte swizzle); thread 0 issues O_blk = P V into TMEM; threads
// rescale-and-add O_blk into their f32 register accumulator.  K and V tiles
// are double-buffered TMA loads issued one block ahead.  The [T, S] score
// matrix never touches HBM.  Causal CTAs skip key blocks above the diagonal
// and are launched heaviest first.
//
// Math: reference src/jax_mlx/sdpa.py:19-31 (softmax(QK^T*scale)V, BTNH
// layout) plus the causal mask JAX applies (keys s > t excluded); replaces
// mlx::fast::scaled_dot_product_attention (src/jax_mlx_pjrt.cpp:4440-4446,
// :8111-8150).
#include <cfloat>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "tc.cuh"

namespace b200 {
namespace {

struct SdpaArgs {
  int B, T, S, N;
  float scale;
  int causal;
  void* o;
  int64_t o_sb, o_st, o_sn;
  float* lse;  // optional [B, N, T]: per-row log2 of sum_s 2^(scale*log2(e)*q.k_s)
  int* err;
};

template <int ES>
struct SdpaCfg {
  static constexpr int E = 128 / ES;               // elements per 128-byte row
  static constexpr int DCH = 64 / E;               // 128-byte chunks per head-dim row
  static constexpr int Q_BYTES = 128 * 64 * ES;    // 128 rows x 64 dims
  static constexpr int KV_BYTES = 128 * 64 * ES;   // 128 keys x 64 dims
  static constexpr int P_BYTES = 128 * 128 * ES;   // 128 rows x 128 keys
  static constexpr int SMEM = Q_BYTES + 4 * KV_BYTES + P_BYTES + 1024 + 256;
};

template <int ES>
__global__ void __launch_bounds__(128, 1)
    sdpa_fwd_tc(const __grid_constant__ CUtensorMap tQ, const __grid_constant__ CUtensorMap tK,
                const __grid_constant__ CUtensorMap tV, SdpaArgs p) {
  pdl_wait();
  using C = SdpaCfg<ES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_BYTES;          // 2 buffers
  uint8_t* sV = sK + 2 * C::KV_BYTES;     // 2 buffers
  uint8_t* sP = sV + 2 * C::KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + C::P_BYTES);
  uint64_t* bar_q = bars;
  uint64_t* bar_k = bars + 1;  // [2]
  uint64_t* bar_v = bars + 3;  // [2]
  uint64_t* bar_s = bars + 5;
  uint64_t* bar_o = bars + 6;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 7);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nq = (p.T + 127) / 128;
  const int qt = p.causal ? nq - 1 - (int)blockIdx.x : (int)blockIdx.x;
  const int n = blockIdx.y, b = blockIdx.z;
  const int t0 = qt * 128;
  const int nkb_all = (p.S + 127) / 128;
  const int nkb = p.causal ? min(nkb_all, (t0 + 127) / 128 + 1) : nkb_all;

  if (tid == 0) {
    for (int i = 0; i < 7; ++i) mbar_init(&bars[i], 1);
    *abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tQ);
    tma_prefetch_desc(&tK);
    tma_prefetch_desc(&tV);
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tS = tmem, tO = tmem + 128;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  auto load_kv = [&](uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int kb) {
    mbar_expect_tx(bar, C::KV_BYTES);
#pragma unroll
    for (int c = 0; c < C::DCH; ++c) tma_load_4d(dst + c * (128 * 128), map, bar, c * C::E, n, kb * 128, b);
  };
  if (tid == 0 && nkb > 0) {
    mbar_expect_tx(bar_q, C::Q_BYTES);
#pragma unroll
    for (int c = 0; c < C::DCH; ++c) tma_load_4d(sQ + c * (128 * 128), &tQ, bar_q, c * C::E, n, t0, b);
    load_kv(sK, &tK, &bar_k[0], 0);
    load_kv(sV, &tV, &bar_v[0], 0);
    if (nkb > 1) {
      load_kv(sK + C::KV_BYTES, &tK, &bar_k[1], 1);
      load_kv(sV + C::KV_BYTES, &tV, &bar_v[1], 1);
    }
  }

  constexpr uint32_t fmt = ES == 4 ? 2u : 1u;
  constexpr uint32_t idesc_s = umma_idesc(fmt, 0, 0, 128, 128);
  constexpr uint32_t idesc_o = umma_idesc(fmt, 0, 1, 64, 128);
  const int row = warp * 32 + lane;
  const int t = t0 + row;
  float o[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) o[i] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;

  for (int j = 0; j < nkb && ok; ++j) {
    const int buf = j & 1;
    if (tid == 0) {
      bool w = true;
      if (j == 0) w = mbar_wait(bar_q, 0, abort, p.err, 201);
      w = w && mbar_wait(&bar_k[buf], (j >> 1) & 1, abort, p.err, 202);
      if (w) {
        tc_fence_after();
        const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK + buf * C::KV_BYTES);
        constexpr int KSTEPS = 64 / (32 / ES);  // head-dim MMA steps (8 tf32, 4 bf16)
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          const uint32_t off = (kk / 4) * (128 * 128) + (kk % 4) * 32;
          const uint64_t ad = umma_desc(q0 + off, 16, 1024), bd = umma_desc(k0 + off, 16, 1024);
          if (ES == 4) umma_tf32(tS, ad, bd, idesc_s, kk != 0);
          else umma_f16(tS, ad, bd, idesc_s, kk != 0);
        }
        umma_commit(bar_s);
      }
    }
    ok = mbar_wait(bar_s, j & 1, abort, p.err, 203);
    ok = __syncthreads_and(ok) != 0;  // block-uniform: no thread may skip a later barrier
    if (!ok) break;
    tc_fence_after();
    // ---- pass 1: row max of this block
    const int kbase = j * 128;
    float bmax = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tmem_ld32(tS + lane_base + c * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int key = kbase + c * 32 + i;
        const bool valid = key < p.S && !(p.causal && key > t);
        if (valid) bmax = fmaxf(bmax, v[i] * p.scale);
      }
    }
    const float m_new = fmaxf(m_run, bmax);
    const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
    // ---- pass 2: P = exp(s*scale - m_new) into shared memory (swizzled K-major)
    float lsum = 0.f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tmem_ld32(tS + lane_base + c * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int key = kbase + c * 32 + i;
        const bool valid = key < p.S && !(p.causal && key > t);
        const float e = valid ? expf(v[i] * p.scale - m_new) : 0.f;
        v[i] = e;
        lsum += e;
      }
      if (ES == 4) {
        // 32 f32 keys = one 128-byte chunk row; 8 units of 4 floats
        uint8_t* prow = sP + c * (128 * 128) + row * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float4 w4 = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
          *reinterpret_cast<float4*>(prow + ((u ^ (row & 7)) * 16)) = w4;
        }
      } else {
        // 32 bf16 keys = half a 128-byte chunk row; 4 units of 8 bf16
        uint8_t* prow = sP + (c / 2) * (128 * 128) + row * 128;
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int u = (c & 1) * 4 + u4;
          uint32_t w[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            __nv_bfloat162 pr = __floats2bfloat162_rn(v[8 * u4 + 2 * h], v[8 * u4 + 2 * h + 1]);
            w[h] = *reinterpret_cast<uint32_t*>(&pr);
          }
          *reinterpret_cast<uint4*>(prow + ((u ^ (row & 7)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    l_run = l_run * alpha + lsum;
    m_run = m_new;
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      if (mbar_wait(&bar_v[buf], (j >> 1) & 1, abort, p.err, 204)) {
        const uint32_t p0 = smem_u32(sP), v0 = smem_u32(sV + buf * C::KV_BYTES);
        constexpr int KSTEPS = 128 / (32 / ES);  // key MMA steps (16 tf32, 8 bf16)
        constexpr uint32_t VSTEP = (32 / ES) * 128;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          const uint64_t ad = umma_desc(p0 + (kk / 4) * (128 * 128) + (kk % 4) * 32, 16, 1024);
          // V is MN-major (head dim contiguous): LBO = stride between 128-byte
          // head-dim chunks, SBO = stride between key-row groups
          const uint64_t bd = ES == 4 ? umma_desc(v0 + kk * VSTEP, 128 * 128, 512, kUmmaSW128Base32)
                                      : umma_desc(v0 + kk * VSTEP, 128 * 128, 1024);
          if (ES == 4) umma_tf32(tO, ad, bd, idesc_o, kk != 0);
          else umma_f16(tO, ad, bd, idesc_o, kk != 0);
        }
        umma_commit(bar_o);
      }
      // K buffer `buf` is free (S of block j finished): prefetch block j+2
      if (j + 2 < nkb) load_kv(sK + buf * C::KV_BYTES, &tK, &bar_k[buf], j + 2);
    }
    ok = mbar_wait(bar_o, j & 1, abort, p.err, 205);
    ok = __syncthreads_and(ok) != 0;  // block-uniform: no thread may skip a later barrier
    if (!ok) break;
    tc_fence_after();
    if (tid == 0 && j + 2 < nkb) load_kv(sV + buf * C::KV_BYTES, &tV, &bar_v[buf], j + 2);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float v[32];
      tmem_ld32(tO + lane_base + c * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * alpha + v[i];
    }
    // the next block's P writes must not overtake this block's TMEM/smem reads
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }

  if (ok && t < p.T) {
    const float inv = 1.f / l_run;
    const int64_t off = (int64_t)b * p.o_sb + (int64_t)t * p.o_st + (int64_t)n * p.o_sn;
    if (ES == 4) {
      float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.o) + off);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        dst[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
    } else {
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.o) + off);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          __nv_bfloat162 pr = __floats2bfloat162_rn(o[8 * i + 2 * h] * inv, o[8 * i + 2 * h + 1] * inv);
          w[h] = *reinterpret_cast<uint32_t*>(&pr);
        }
        dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort && tid == 0) {
    const uint64_t t1 = globaltimer();
    while (globaltimer() - t1 < 2000000ull) {
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------------------
// f32 inputs, 3xTF32: every operand is split into tf32 hi and lo parts in shared
// memory and each product is formed as lo*hi + hi*lo + hi*hi, which keeps the
// scores and the output at f32-level accuracy (plain TF32 truncation leaves
// ~1e-3 relative error in the logits, which exp() passes on).  Key blocks of 64
// so that Q, K (double-buffered), V and P with their lo parts fit in 224 KB.
constexpr int X3_KEYS = 64;

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
__device__ __forceinline__ void split16(uint8_t* tile, uint8_t* lo, int bytes, int tid) {
  for (int off = tid * 16; off < bytes; off += 128 * 16) {
    float4 v = *reinterpret_cast<float4*>(tile + off);
    float4 h = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
    *reinterpret_cast<float4*>(tile + off) = h;
    *reinterpret_cast<float4*>(lo + off) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
  }
}

struct X3Cfg {
  static constexpr int Q = 128 * 64 * 4;        // 32 KB (two 16 KB head-dim chunks)
  static constexpr int KV = X3_KEYS * 64 * 4;   // 16 KB (two 8 KB chunks)
  static constexpr int P = 128 * X3_KEYS * 4;   // 32 KB (two 16 KB key chunks)
  // Q, Qlo | K0, K0lo, K1, K1lo | V, Vlo | P, Plo
  static constexpr int SMEM = 2 * Q + 4 * KV + 2 * KV + 2 * P + 1024 + 256;
};

__global__ void __launch_bounds__(128, 1)
    sdpa_fwd_tc_x3(const __grid_constant__ CUtensorMap tQ, const __grid_constant__ CUtensorMap tK,
                   const __grid_constant__ CUtensorMap tV, SdpaArgs p) {
  pdl_wait();
  using C = X3Cfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;
  uint8_t* sQlo = sQ + C::Q;
  uint8_t* sK = sQlo + C::Q;                // buffer b: sK + b * 2*KV, lo at +KV
  uint8_t* sV = sK + 4 * C::KV;             // V, then Vlo at +KV
  uint8_t* sP = sV + 2 * C::KV;             // P, then Plo at +P
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::P);
  uint64_t* bar_q = bars;
  uint64_t* bar_k = bars + 1;  // [2]
  uint64_t* bar_v = bars + 3;
  uint64_t* bar_s = bars + 4;
  uint64_t* bar_o = bars + 5;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nq = (p.T + 127) / 128;
  const int qt = p.causal ? nq - 1 - (int)blockIdx.x : (int)blockIdx.x;
  const int n = blockIdx.y, b = blockIdx.z;
  const int t0 = qt * 128;
  const int nkb_all = (p.S + X3_KEYS - 1) / X3_KEYS;
  const int nkb = p.causal ? min(nkb_all, (t0 + 127) / X3_KEYS + 1) : nkb_all;

  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(&bars[i], 1);
    *abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tQ);
    tma_prefetch_desc(&tK);
    tma_prefetch_desc(&tV);
  }
  if (warp == 0) {
    tmem_alloc(tslot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tS = tmem, tO = tmem + 64;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  auto load_k = [&](int buf, int kb) {
    uint64_t* bar = &bar_k[buf];
    mbar_expect_tx(bar, C::KV);
    for (int c = 0; c < 2; ++c)
      tma_load_4d(sK + buf * 2 * C::KV + c * (X3_KEYS * 128), &tK, bar, c * 32, n, kb * X3_KEYS, b);
  };
  auto load_v = [&](int kb) {
    mbar_expect_tx(bar_v, C::KV);
    for (int c = 0; c < 2; ++c)
      tma_load_4d(sV + c * (X3_KEYS * 128), &tV, bar_v, c * 32, n, kb * X3_KEYS, b);
  };
  if (tid == 0 && nkb > 0) {
    mbar_expect_tx(bar_q, C::Q);
    for (int c = 0; c < 2; ++c) tma_load_4d(sQ + c * (128 * 128), &tQ, bar_q, c * 32, n, t0, b);
    load_k(0, 0);
    if (nkb > 1) load_k(1, 1);
    load_v(0);
  }
  constexpr uint32_t idesc_s = umma_idesc(2, 0, 0, X3_KEYS, 128);
  constexpr uint32_t idesc_o = umma_idesc(2, 0, 1, 64, 128);
  const int row = warp * 32 + lane;
  const int t = t0 + row;
  float o[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) o[i] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = nkb > 0;
  if (ok) {
    ok = mbar_wait(bar_q, 0, abort, p.err, 211);
    ok = __syncthreads_and(ok) != 0;
    if (ok) split16(sQ, sQlo, C::Q, tid);
  }

  for (int j = 0; j < nkb && ok; ++j) {
    const int buf = j & 1;
    uint8_t* kh = sK + buf * 2 * C::KV;
    uint8_t* kl = kh + C::KV;
    ok = mbar_wait(&bar_k[buf], (j >> 1) & 1, abort, p.err, 212);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    split16(kh, kl, C::KV, tid);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t qh0 = smem_u32(sQ), ql0 = smem_u32(sQlo), kh0 = smem_u32(kh), kl0 = smem_u32(kl);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {  // head dim: 8 steps of 8
        const uint32_t qo = (kk / 4) * (128 * 128) + (kk % 4) * 32;
        const uint32_t ko = (kk / 4) * (X3_KEYS * 128) + (kk % 4) * 32;
        const uint64_t qh = umma_desc(qh0 + qo, 16, 1024), ql = umma_desc(ql0 + qo, 16, 1024);
        const uint64_t kdh = umma_desc(kh0 + ko, 16, 1024), kdl = umma_desc(kl0 + ko, 16, 1024);
        umma_tf32(tS, ql, kdh, idesc_s, kk != 0);
        umma_tf32(tS, qh, kdl, idesc_s, 1);
        umma_tf32(tS, qh, kdh, idesc_s, 1);
      }
      umma_commit(bar_s);
    }
    ok = mbar_wait(bar_s, j & 1, abort, p.err, 213);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    tc_fence_after();
    // K buffer `buf` is free again (S of block j finished): prefetch block j+2
    if (tid == 0 && j + 2 < nkb) load_k(buf, j + 2);
    const int kbase = j * X3_KEYS;
    float sv[64];
    tmem_ld32(tS + lane_base, sv);
    tmem_ld32(tS + lane_base + 32, sv + 32);
    float bmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const int key = kbase + i;
      const bool valid = key < p.S && !(p.causal && key > t);
      sv[i] = valid ? sv[i] * p.scale : -INFINITY;
      bmax = fmaxf(bmax, sv[i]);
    }
    const float m_new = fmaxf(m_run, bmax);
    const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
    float lsum = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const float e = sv[i] == -INFINITY ? 0.f : expf(sv[i] - m_new);
      sv[i] = e;
      lsum += e;
    }
    l_run = l_run * alpha + lsum;
    m_run = m_new;
    // P hi/lo into shared memory (K-major over keys, 128-byte swizzle)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint8_t* ph = sP + c * (128 * 128) + row * 128;
      uint8_t* pl = ph + C::P;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float* e = sv + c * 32 + 4 * u;
        float4 h = make_float4(tf32_rna(e[0]), tf32_rna(e[1]), tf32_rna(e[2]), tf32_rna(e[3]));
        const int sw = (u ^ (row & 7)) * 16;
        *reinterpret_cast<float4*>(ph + sw) = h;
        *reinterpret_cast<float4*>(pl + sw) = make_float4(e[0] - h.x, e[1] - h.y, e[2] - h.z, e[3] - h.w);
      }
    }
    ok = mbar_wait(bar_v, j & 1, abort, p.err, 214);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    split16(sV, sV + C::KV, C::KV, tid);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ph0 = smem_u32(sP), pl0 = smem_u32(sP + C::P);
      const uint32_t vh0 = smem_u32(sV), vl0 = smem_u32(sV + C::KV);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {  // keys: 8 steps of 8
        const uint32_t po = (kk / 4) * (128 * 128) + (kk % 4) * 32;
        const uint64_t pdh = umma_desc(ph0 + po, 16, 1024), pdl = umma_desc(pl0 + po, 16, 1024);
        // V MN-major (head dim contiguous): LBO = 8 KB between 32-dim chunks,
        // SBO = 512 B between 4-key row groups (tf32 layout)
        const uint64_t vdh = umma_desc(vh0 + kk * 1024, X3_KEYS * 128, 512, kUmmaSW128Base32);
        const uint64_t vdl = umma_desc(vl0 + kk * 1024, X3_KEYS * 128, 512, kUmmaSW128Base32);
        umma_tf32(tO, pdl, vdh, idesc_o, kk != 0);
        umma_tf32(tO, pdh, vdl, idesc_o, 1);
        umma_tf32(tO, pdh, vdh, idesc_o, 1);
      }
      umma_commit(bar_o);
    }
    ok = mbar_wait(bar_o, j & 1, abort, p.err, 215);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    tc_fence_after();
    if (tid == 0 && j + 1 < nkb) load_v(j + 1);  // V buffer free: PV of block j finished
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float v[32];
      tmem_ld32(tO + lane_base + c * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * alpha + v[i];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }

  if (ok && t < p.T) {
    const float inv = 1.f / l_run;
    const int64_t off = (int64_t)b * p.o_sb + (int64_t)t * p.o_st + (int64_t)n * p.o_sn;
    float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.o) + off);
#pragma unroll
    for (int i = 0; i < 16; ++i)
      dst[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
  }
  tc_fence_before();
  __syncthreads();
  if (*abort && tid == 0) {
    const uint64_t t1 = globaltimer();
    while (globaltimer() - t1 < 2000000ull) {
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ---------------------------------------------------------------------------
// Warp-specialized attention forward, head dim 64, key blocks of 64.
//
// One CTA = 128 query rows of one (batch, head), 448 threads in four roles:
//   warps 0-7  softmax: warp w owns TMEM lane quarter w % 4 (32 query rows)
//              and half w / 4 of each key block and of the head dim; reads S_j
//              from TMEM, exchanges the row max with its partner warp, keeps
//              the online max / sum in f32, writes P_j as bf16 into TMEM, and
//              folds the previous block's P V product (TMEM) into its f32 half
//              row of O held in registers;
//   warp 8     TMA: Q once, then K_j / V_j into a three-slot ring;
//   warp 9     MMA issue: S_j = Q K_j^T (A = Q in shared memory) into one of two
//              TMEM S buffers, then O_{j-1} = P_{j-1} V_{j-1} with A = P read
//              straight from TMEM into one of two TMEM O buffers, so the tensor
//              core works on block j while the softmax warps work on block j-1;
//   warps 10-13 (f32 inputs) split each f32 tile into bf16 hi and lo parts.
// f32 inputs run every product as three bf16 MMAs, hi*hi + hi*lo + lo*hi
// (the dropped lo*lo term is ~2^-16 relative), on Q, K, V and P; bf16 inputs
// run one.  Shared-memory operand tiles are 128-byte rows with the 16-byte
// unit swizzle (unit ^ row % 8): K-major for Q and K, MN-major for V.
template <bool X3>
struct WsCfg {
  static constexpr int QB = 128 * 128;   // bf16 Q tile: 128 rows x 128 B
  static constexpr int KB = 64 * 128;    // bf16 K or V tile: 64 keys x 128 B
  static constexpr int PARTS = X3 ? 2 : 1;
  static constexpr int SLOTS = 3;                                  // K/V ring depth
  static constexpr int Q_OFF = 0;                                  // Q hi [, lo]
  static constexpr int KV_OFF = Q_OFF + PARTS * QB;                // slot s: K hi, [K lo,] V hi [, V lo]
  static constexpr int KV_SLOT = 2 * PARTS * KB;
  // f32 staging (X3): K and V of two blocks (buffer b of K at ST_OFF + b * 2 * 16 KB,
  // V 16 KB after it), so block j+1's loads land while block j is being split
  static constexpr int ST_OFF = KV_OFF + SLOTS * KV_SLOT;
  static constexpr int ST_BYTES = X3 ? 2 * 2 * 64 * 256 : 0;
  static constexpr int QST_OFF = KV_OFF + 2 * KV_SLOT;             // f32 Q staging aliases K/V slot 2
  static constexpr int RED_OFF = ST_OFF + ST_BYTES;                // softmax max / sum exchange
  static constexpr int BAR_OFF = RED_OFF + 2 * 2 * 128 * 4;
  static constexpr int SMEM = BAR_OFF + 512 + 1024;
  static_assert(!X3 || KV_SLOT >= 128 * 256, "f32 Q staging must fit in one K/V slot");
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// Split 4 f32 into bf16 hi (rounded) and lo (rounded residual), 8 bytes each.
__device__ __forceinline__ void split4(float4 x, uint2& hi, uint2& lo) {
  __nv_bfloat162 h0 = __floats2bfloat162_rn(x.x, x.y), h1 = __floats2bfloat162_rn(x.z, x.w);
  const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
  hi = make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
  lo = make_uint2(pack_bf16x2(x.x - f0.x, x.y - f0.y), pack_bf16x2(x.z - f1.x, x.w - f1.y));
}
// f32 staging tile (rows x 64, two 128-byte-swizzled chunks of 32 columns,
// chunk c at c * rows * 128) -> bf16 hi / lo tiles (rows x 128 B, swizzled).
__device__ __forceinline__ void split_rows(const uint8_t* st, uint8_t* hi, uint8_t* lo, int rows,
                                           int ctid) {
  for (int f = ctid; f < rows * 16; f += 128) {
    const int r = f >> 4, c = (f >> 3) & 1, u = f & 7;
    const float4 x = *reinterpret_cast<const float4*>(st + c * rows * 128 + r * 128 + ((u ^ (r & 7)) << 4));
    uint2 h, l;
    split4(x, h, l);
    const int U = c * 4 + (u >> 1);
    const int off = r * 128 + ((U ^ (r & 7)) << 4) + (u & 1) * 8;
    *reinterpret_cast<uint2*>(hi + off) = h;
    *reinterpret_cast<uint2*>(lo + off) = l;
  }
}

// Thread roles: warps 0-7 softmax, warp 8 TMA, warp 9 MMA issue, and for f32
// inputs warps 10-13 split (448 threads, 512 TMEM columns, one CTA per SM).
// bf16 inputs run 320 threads in 256 TMEM columns with one O buffer, so that
// two CTAs share an SM and one's softmax hides the other's waits.
template <bool X3>
struct WsShape {
  static constexpr int THREADS = X3 ? 448 : 320;
  static constexpr int MIN_CTAS = X3 ? 1 : 2;
  static constexpr uint32_t TMEM_COLS = X3 ? 512 : 256;
  static constexpr int NOB = X3 ? 2 : 1;  // O buffers in TMEM
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool X3>
__global__ void __launch_bounds__(WsShape<X3>::THREADS, WsShape<X3>::MIN_CTAS)
    sdpa_fwd_ws(const __grid_constant__ CUtensorMap tQ, const __grid_constant__ CUtensorMap tK,
                const __grid_constant__ CUtensorMap tV, SdpaArgs p) {
  pdl_wait();
  using C = WsCfg<X3>;
  constexpr int NS = C::SLOTS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* q_hi = smem + C::Q_OFF;
  uint8_t* q_lo = q_hi + C::QB;
  auto k_hi = [&](int s) { return smem + C::KV_OFF + s * C::KV_SLOT; };
  auto k_lo = [&](int s) { return smem + C::KV_OFF + s * C::KV_SLOT + C::KB; };
  auto v_hi = [&](int s) { return smem + C::KV_OFF + s * C::KV_SLOT + C::PARTS * C::KB; };
  auto v_lo = [&](int s) { return smem + C::KV_OFF + s * C::KV_SLOT + 3 * C::KB; };
  auto k_st = [&](int bf) { return smem + C::ST_OFF + bf * 2 * 64 * 256; };
  auto v_st = [&](int bf) { return smem + C::ST_OFF + bf * 2 * 64 * 256 + 64 * 256; };
  uint8_t* q_st = smem + C::QST_OFF;
  float* red = reinterpret_cast<float*>(smem + C::RED_OFF);  // [2 block parities][2 halves][128 rows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* q_ready = bars + 1;
  uint64_t* kv_full = bars + 2;    // [3] K/V slot loaded (bf16 inputs)
  uint64_t* kv_conv = bars + 5;    // [3] K/V slot split (f32 inputs)
  uint64_t* kv_free = bars + 8;    // [3] K/V slot consumed by the MMAs
  uint64_t* s_full = bars + 11;    // [2]
  uint64_t* s_free = bars + 13;    // [2]
  uint64_t* p_full = bars + 15;    // [2]
  uint64_t* o_full = bars + 17;    // [2]
  uint64_t* ob_free = bars + 19;   // [2]
  uint64_t* mx_bar = bars + 21;    // [4 quarters][2]: both halves' block maxima written
  uint64_t* l_bar = bars + 29;     // [4 quarters]: both halves' row sums written
  uint64_t* kst_full = bars + 33;  // [2] f32 K staging buffer loaded
  uint64_t* vst_full = bars + 35;  // [2] f32 V staging buffer loaded
  uint64_t* kst_used = bars + 37;  // [2] f32 K staging buffer split (count 4 warps)
  uint64_t* vst_used = bars + 39;  // [2] f32 V staging buffer split
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 41);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // one-dimensional grid, query tile slowest: with a causal mask every CTA
  // of the first (N * B) holds a last (heaviest) query tile, and lighter tiles
  // follow, so SMs that finish early pick up the light work (longest first)
  const int nq = (p.T + 127) / 128;
  const int nb = p.N * p.B;
  const int tile = (int)blockIdx.x / nb, nbi = (int)blockIdx.x % nb;
  const int qt = p.causal ? nq - 1 - tile : tile;
  const int n = nbi % p.N, b = nbi / p.N;
  const int t0 = qt * 128;
  const int nkb_all = (p.S + 63) / 64;
  const int nkb = p.causal ? min(nkb_all, (t0 + 127) / 64 + 1) : nkb_all;

  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_ready, 4);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_conv[i], 4);
      mbar_init(&kv_free[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 8);
      mbar_init(&p_full[i], 8);
      mbar_init(&o_full[i], 1);
      mbar_init(&ob_free[i], 8);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&mx_bar[i], 2);
    for (int i = 0; i < 4; ++i) mbar_init(&l_bar[i], 2);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kst_full[i], 1);
      mbar_init(&vst_full[i], 1);
      mbar_init(&kst_used[i], 4);
      mbar_init(&vst_used[i], 4);
    }
    *abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, WsShape<X3>::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // TMEM columns (f32 / packed bf16x2): S buffers at 0 and 64; f32 inputs: O
  // buffers at 128 and 192, P buffers at 256 and 320 (hi in the first 32
  // columns, lo in the last 32); bf16 inputs: one O buffer at 128, P buffers
  // (32 packed columns) at 192 and 224
  constexpr int NOB = WsShape<X3>::NOB;
  auto tS = [&](int s) { return tmem + (uint32_t)(s * 64); };
  auto tO = [&](int s) { return tmem + 128u + (uint32_t)(s * 64); };
  auto tP = [&](int s) { return X3 ? tmem + 256u + (uint32_t)(s * 64) : tmem + 192u + (uint32_t)(s * 32); };

  if (warp == 8) {
    if (lane == 0 && nkb > 0) {  // ---- TMA producer
      tma_prefetch_desc(&tQ);
      tma_prefetch_desc(&tK);
      tma_prefetch_desc(&tV);
      if (X3) {
        mbar_expect_tx(q_full, 128 * 64 * 4);
        for (int c = 0; c < 2; ++c) tma_load_4d(q_st + c * 128 * 128, &tQ, q_full, c * 32, n, t0, b);
      } else {
        mbar_expect_tx(q_full, 128 * 64 * 2);
        tma_load_4d(q_hi, &tQ, q_full, 0, n, t0, b);
      }
      for (int j = 0; j < nkb; ++j) {
        const int ks = j % NS, kuse = j / NS;
        if (X3) {
          // two f32 staging buffers each for K and V: block j's K may land in
          // buffer j % 2 once block j-2's K has been split out of it
          const int bf = j & 1;
          if (j >= 2 && !mbar_wait(&kst_used[bf], ((j - 2) >> 1) & 1, abort, p.err, 211)) break;
          mbar_expect_tx(&kst_full[bf], 64 * 64 * 4);
          for (int c = 0; c < 2; ++c)
            tma_load_4d(k_st(bf) + c * 64 * 128, &tK, &kst_full[bf], c * 32, n, j * 64, b);
          if (j >= 2 && !mbar_wait(&vst_used[bf], ((j - 2) >> 1) & 1, abort, p.err, 210)) break;
          mbar_expect_tx(&vst_full[bf], 64 * 64 * 4);
          for (int c = 0; c < 2; ++c)
            tma_load_4d(v_st(bf) + c * 64 * 128, &tV, &vst_full[bf], c * 32, n, j * 64, b);
        } else {
          if (j >= NS && !mbar_wait(&kv_free[ks], (kuse - 1) & 1, abort, p.err, 211)) break;
          mbar_expect_tx(&kv_full[ks], 2 * 64 * 64 * 2);
          tma_load_4d(k_hi(ks), &tK, &kv_full[ks], 0, n, j * 64, b);
          tma_load_4d(v_hi(ks), &tV, &kv_full[ks], 0, n, j * 64, b);
        }
      }
    }
  } else if (warp == 9) {
    if (lane == 0 && nkb > 0) {  // ---- MMA issuer
      constexpr uint32_t idesc_s = umma_idesc(1u, 0, 0, 64, 128);
      constexpr uint32_t idesc_o = umma_idesc(1u, 0, 1, 64, 128);
      bool ok = mbar_wait(X3 ? q_ready : q_full, 0, abort, p.err, 212);
      for (int j = 0; ok && j <= nkb; ++j) {
        if (j < nkb) {
          const int ks = j % NS, kuse = j / NS, sb = j & 1, suse = j >> 1;
          ok = mbar_wait(X3 ? &kv_conv[ks] : &kv_full[ks], kuse & 1, abort, p.err, 213);
          if (ok && j >= 2) ok = mbar_wait(&s_free[sb], (suse - 1) & 1, abort, p.err, 214);
          if (!ok) break;
          tc_fence_after();
          const uint32_t qh = smem_u32(q_hi), ql = smem_u32(q_lo);
          const uint32_t kh = smem_u32(k_hi(ks)), kl = smem_u32(k_lo(ks));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t off = kk * 32;
            umma_f16(tS(sb), umma_desc(qh + off, 16, 1024), umma_desc(kh + off, 16, 1024), idesc_s, kk != 0);
            if (X3) {
              umma_f16(tS(sb), umma_desc(qh + off, 16, 1024), umma_desc(kl + off, 16, 1024), idesc_s, 1);
              umma_f16(tS(sb), umma_desc(ql + off, 16, 1024), umma_desc(kh + off, 16, 1024), idesc_s, 1);
            }
          }
          umma_commit(&s_full[sb]);
        }
        if (j >= 1) {
          const int jj = j - 1, ks1 = jj % NS, b1 = jj & 1, use1 = jj >> 1;
          const int ob = jj % NOB, ouse = jj / NOB;  // O buffer of block jj and its use count
          ok = mbar_wait(&p_full[b1], use1 & 1, abort, p.err, 215);
          if (ok && jj >= NOB) ok = mbar_wait(&ob_free[ob], (ouse - 1) & 1, abort, p.err, 216);
          if (!ok) break;
          tc_fence_after();
          const uint32_t vh = smem_u32(v_hi(ks1)), vl = smem_u32(v_lo(ks1));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // P in TMEM: 16 keys = 8 packed columns; V: MN-major, 16 keys = 16 rows of 128 B
            const uint32_t pa = tP(b1) + kk * 8, vb = kk * 2048;
            umma_f16_ts(tO(ob), pa, umma_desc(vh + vb, 8192, 1024), idesc_o, kk != 0);
            if (X3) {
              umma_f16_ts(tO(ob), pa, umma_desc(vl + vb, 8192, 1024), idesc_o, 1);
              umma_f16_ts(tO(ob), pa + 32, umma_desc(vh + vb, 8192, 1024), idesc_o, 1);
            }
          }
          umma_commit(&o_full[ob]);
          umma_commit(&kv_free[ks1]);
        }
      }
    }
  } else if (warp >= 10) {
    if (X3 && nkb > 0) {  // ---- f32 -> bf16 hi/lo split
      const int ctid = tid - 320;
      bool ok = mbar_wait(q_full, 0, abort, p.err, 217);
      if (__all_sync(0xffffffffu, ok)) {
        split_rows(q_st, q_hi, q_lo, 128, ctid);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_ready);
        for (int j = 0; j < nkb; ++j) {
          const int ks = j % NS, kuse = j / NS;
          ok = j < NS || mbar_wait(&kv_free[ks], (kuse - 1) & 1, abort, p.err, 219);
          const int bf = j & 1;
          ok = ok && mbar_wait(&kst_full[bf], (j >> 1) & 1, abort, p.err, 218);
          if (!__all_sync(0xffffffffu, ok)) break;
          split_rows(k_st(bf), k_hi(ks), k_lo(ks), 64, ctid);
          __syncwarp();
          if (lane == 0) mbar_arrive(&kst_used[bf]);
          ok = mbar_wait(&vst_full[bf], (j >> 1) & 1, abort, p.err, 224);
          if (!__all_sync(0xffffffffu, ok)) break;
          split_rows(v_st(bf), v_hi(ks), v_lo(ks), 64, ctid);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&vst_used[bf]);
            mbar_arrive(&kv_conv[ks]);
          }
        }
      }
    }
  } else {  // ---- warps 0-7: softmax and output
    const int q = warp & 3, h = warp >> 2;  // TMEM lane quarter, key / head-dim half
    const int row = q * 32 + lane;
    const int t = t0 + row;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const float sl2 = p.scale * 1.4426950408889634f;  // scale * log2(e)
    float o[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, m_acc = -INFINITY;
    float m_hist0 = -INFINITY, m_hist1 = -INFINITY;
    bool ok = true;
    auto fold = [&](int jj) {  // o = o * 2^(m_acc - m_jj) + (P_jj V_jj)[this half]
      const int s1 = jj & 1, ob = jj % NOB;
      bool w = mbar_wait(&o_full[ob], (jj / NOB) & 1, abort, p.err, 220);
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
      const float mj = s1 ? m_hist1 : m_hist0;
      const float a = m_acc == -INFINITY ? 0.f : ex2(m_acc - mj);
      float v[32];
      tmem_ld32(tO(ob) + lane_base + h * 32, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ob_free[ob]);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = fmaf(o[i], a, v[i]);
      m_acc = mj;
      return true;
    };
    for (int j = 0; j < nkb; ++j) {
      const int s = j & 1, use = j >> 1;
      bool w = mbar_wait(&s_full[s], use & 1, abort, p.err, 221);
      if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
      tc_fence_after();
      float v[32];
      tmem_ld32(tS(s) + lane_base + h * 32, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[s]);  // S_j is in registers
      const int kbase = j * 64 + h * 32;
      const bool need_mask = kbase + 32 > p.S || (p.causal && kbase + 31 > t0);
      if (need_mask) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = kbase + i;
          if (key >= p.S || (p.causal && key > t)) v[i] = -INFINITY;
        }
      }
      float bmax = v[0];
#pragma unroll
      for (int i = 1; i < 32; ++i) bmax = fmaxf(bmax, v[i]);
      // row max over both halves: exchange through shared memory; the mbarrier
      // of this quarter and block parity completes once both warps have written
      // (a later reuse of the buffer happens only after the partner's next
      // arrival, i.e. after it has read this one)
      float* rb = red + (j & 1) * 256;
      rb[h * 128 + row] = bmax;
      __syncwarp();
      if (lane == 0) mbar_arrive(&mx_bar[q * 2 + s]);
      w = mbar_wait(&mx_bar[q * 2 + s], use & 1, abort, p.err, 222);
      if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
      bmax = fmaxf(rb[row], rb[128 + row]);
      const float m_new = fmaxf(m_run, bmax * sl2);
      const float alpha = m_run == -INFINITY ? 0.f : ex2(m_run - m_new);
      const float mo = m_new == -INFINITY ? 0.f : m_new;
      float lsum = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float e = ex2(fmaf(v[i], sl2, -mo));  // masked: 2^-inf = 0
        v[i] = e;
        lsum += e;
      }
      // P_j half row -> TMEM (packed bf16 pairs; hi, and lo for f32 inputs).
      // P buffer s was last read by P_{j-2} V_{j-2}, folded before this block.
      uint32_t ph[16], pl[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        __nv_bfloat162 hh = __floats2bfloat162_rn(v[2 * c], v[2 * c + 1]);
        ph[c] = *reinterpret_cast<uint32_t*>(&hh);
        if (X3) {
          const float2 f = __bfloat1622float2(hh);
          pl[c] = pack_bf16x2(v[2 * c] - f.x, v[2 * c + 1] - f.y);
        }
      }
      tmem_st16(tP(s) + lane_base + h * 16, ph);
      if (X3) tmem_st16(tP(s) + lane_base + 32 + h * 16, pl);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
      l_run = l_run * alpha + lsum;
      m_run = m_new;
      if (s) m_hist1 = m_new; else m_hist0 = m_new;
      if (j >= 1 && !fold(j - 1)) { ok = false; break; }
    }
    if (ok && nkb > 0) ok = fold(nkb - 1);
    // row sum over both halves
    // (the exchange buffer of parity nkb & 1 was last read for block nkb - 2,
    // before the partner's arrival for block nkb - 1 that this warp waited on)
    float* lb = red + (nkb & 1) * 256;
    if (ok) {
      lb[h * 128 + row] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(&l_bar[q]);
      const bool w = mbar_wait(&l_bar[q], 0, abort, p.err, 223);
      ok = __all_sync(0xffffffffu, w) != 0;
    }
    if (ok && t < p.T) {
      const float lsum = lb[row] + lb[128 + row];
      const float inv = 1.f / lsum;
      if (p.lse && h == 0) p.lse[((int64_t)b * p.N + n) * p.T + t] = m_run + log2f(lsum);
      const int64_t off = (int64_t)b * p.o_sb + (int64_t)t * p.o_st + (int64_t)n * p.o_sn + h * 32;
      if (X3) {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.o) + off);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.o) + off);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[i] = make_uint4(pack_bf16x2(o[8 * i] * inv, o[8 * i + 1] * inv),
                              pack_bf16x2(o[8 * i + 2] * inv, o[8 * i + 3] * inv),
                              pack_bf16x2(o[8 * i + 4] * inv, o[8 * i + 5] * inv),
                              pack_bf16x2(o[8 * i + 6] * inv, o[8 * i + 7] * inv));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort && tid == 0) {
    const uint64_t t1 = globaltimer();
    while (globaltimer() - t1 < 2000000ull) {
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, WsShape<X3>::TMEM_COLS);
  }
}

template <bool X3>
int launch_ws(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t T,
              int64_t S, int64_t N, const int64_t* st, float scale, int causal, cudaStream_t s,
              float* lse = nullptr) {
  using C = WsCfg<X3>;
  constexpr int ES = X3 ? 4 : 2;
  constexpr uint32_t inner = X3 ? 32 : 64;  // 128-byte rows
  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[4] = {64, (uint64_t)N, (uint64_t)T, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)(st[2] * ES), (uint64_t)(st[1] * ES), (uint64_t)(st[0] * ES)};
    const uint32_t box[4] = {inner, 1, 128, 1};
    if (int rc = make_tmap(&tq, q, 4, dims, str, box, ES)) return rc;
  }
  {
    const uint64_t dims[4] = {64, (uint64_t)N, (uint64_t)S, (uint64_t)B};
    const uint32_t box[4] = {inner, 1, 64, 1};
    const uint64_t sk[3] = {(uint64_t)(st[5] * ES), (uint64_t)(st[4] * ES), (uint64_t)(st[3] * ES)};
    if (int rc = make_tmap(&tk, k, 4, dims, sk, box, ES)) return rc;
    const uint64_t sv[3] = {(uint64_t)(st[8] * ES), (uint64_t)(st[7] * ES), (uint64_t)(st[6] * ES)};
    if (int rc = make_tmap(&tv, v, 4, dims, sv, box, ES)) return rc;
  }
  SdpaArgs a{};
  a.B = (int)B;
  a.T = (int)T;
  a.S = (int)S;
  a.N = (int)N;
  a.scale = scale;
  a.causal = causal;
  a.o = o;
  a.o_sb = st[9];
  a.o_st = st[10];
  a.o_sn = st[11];
  a.lse = lse;
  a.err = device_error_word();
  if (!a.err) return set_error(B200_ERR_CUDA, "could not allocate the device error word");
  if (int rc = allow_dynamic_smem((const void*)sdpa_fwd_ws<X3>, C::SMEM, "sdpa_fwd_ws")) return rc;
  const int64_t ctas = (T + 127) / 128 * N * B;
  if (ctas >= (1ll << 31)) return set_error(B200_ERR_INVALID, "sdpa: too many query tiles");
  B200_LAUNCH(sdpa_fwd_ws<X3>, dim3((unsigned)ctas), dim3(WsShape<X3>::THREADS), C::SMEM, s, tq, tk, tv, a);
  return B200_OK;
}

// SIMT fallback for shapes the tensor-core kernel does not take (head dim !=
// 64, unaligned strides): one block per (query row, head, batch), scores in
// shared memory, exact f32 arithmetic.
template <typename T>
__global__ void __launch_bounds__(128)
    sdpa_fwd_simt(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                  T* __restrict__ o, int S, int D, const int64_t* __restrict__ st, float scale,
                  int causal) {
  pdl_wait();
  extern __shared__ float sc[];  // S scores, then D query values
  float* qv = sc + S;
  const int t = blockIdx.x, n = blockIdx.y, b = blockIdx.z;
  const T* qr = q + b * st[0] + t * st[1] + n * st[2];
  for (int d = threadIdx.x; d < D; d += blockDim.x) qv[d] = Io<T>::to_f(qr[d]);
  __syncthreads();
  const int send = causal ? min(S, t + 1) : S;
  for (int s = threadIdx.x; s < send; s += blockDim.x) {
    const T* kr = k + b * st[3] + s * st[4] + n * st[5];
    float acc = 0.f;
    for (int d = 0; d < D; ++d) acc = fmaf(qv[d], Io<T>::to_f(kr[d]), acc);
    sc[s] = acc * scale;
  }
  __syncthreads();
  __shared__ float red[32];
  float mx = -INFINITY;
  for (int s = threadIdx.x; s < send; s += blockDim.x) mx = fmaxf(mx, sc[s]);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = -INFINITY;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float sum = 0.f;
  for (int s = threadIdx.x; s < send; s += blockDim.x) {
    const float e = expf(sc[s] - mx);
    sc[s] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  sum = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) sum += red[i];
  const float inv = 1.f / sum;
  T* orow = o + b * st[9] + t * st[10] + n * st[11];
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < send; ++s) acc = fmaf(sc[s], Io<T>::to_f(v[b * st[6] + s * st[7] + n * st[8] + d]), acc);
    orow[d] = Io<T>::from_f(acc * inv);
  }
}

template <int ES>
int launch_tc(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t T,
              int64_t S, int64_t N, const int64_t* st, float scale, int causal, cudaStream_t s) {
  using C = SdpaCfg<ES>;
  CUtensorMap tq, tk, tv;
  const uint32_t box[4] = {(uint32_t)C::E, 1, 128, 1};
  {
    const uint64_t dims[4] = {64, (uint64_t)N, (uint64_t)T, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)(st[2] * ES), (uint64_t)(st[1] * ES), (uint64_t)(st[0] * ES)};
    if (int rc = make_tmap(&tq, q, 4, dims, str, box, ES)) return rc;
  }
  {
    const uint64_t dims[4] = {64, (uint64_t)N, (uint64_t)S, (uint64_t)B};
    const uint64_t sk[3] = {(uint64_t)(st[5] * ES), (uint64_t)(st[4] * ES), (uint64_t)(st[3] * ES)};
    if (int rc = make_tmap(&tk, k, 4, dims, sk, box, ES)) return rc;
    const uint64_t sv[3] = {(uint64_t)(st[8] * ES), (uint64_t)(st[7] * ES), (uint64_t)(st[6] * ES)};
    if (int rc = make_tmap(&tv, v, 4, dims, sv, box, ES, /*atom32=*/ES == 4)) return rc;
  }
  SdpaArgs a{};
  a.B = (int)B;
  a.T = (int)T;
  a.S = (int)S;
  a.N = (int)N;
  a.scale = scale;
  a.causal = causal;
  a.o = o;
  a.o_sb = st[9];
  a.o_st = st[10];
  a.o_sn = st[11];
  a.err = device_error_word();
  if (!a.err) return set_error(B200_ERR_CUDA, "could not allocate the device error word");
  if (int rc = allow_dynamic_smem((const void*)sdpa_fwd_tc<ES>, C::SMEM, "sdpa_fwd_tc")) return rc;
  dim3 grid((unsigned)((T + 127) / 128), (unsigned)N, (unsigned)B);
  B200_LAUNCH(sdpa_fwd_tc<ES>, grid, dim3(128), C::SMEM, s, tq, tk, tv, a);
  return B200_OK;
}

int launch_x3(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t T,
              int64_t S, int64_t N, const int64_t* st, float scale, int causal, cudaStream_t s) {
  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[4] = {64, (uint64_t)N, (uint64_t)T, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)(st[2] * 4), (uint64_t)(st[1] * 4), (uint64_t)(st[0] * 4)};
    const uint32_t box[4] = {32, 1, 128, 1};
    if (int rc = make_tmap(&tq, q, 4, dims, str, box, 4)) return rc;
  }
  {
    const uint64_t dims[4] = {64, (uint64_t)N, (uint64_t)S, (uint64_t)B};
    const uint32_t box[4] = {32, 1, X3_KEYS, 1};
    const uint64_t sk[3] = {(uint64_t)(st[5] * 4), (uint64_t)(st[4] * 4), (uint64_t)(st[3] * 4)};
    if (int rc = make_tmap(&tk, k, 4, dims, sk, box, 4)) return rc;
    const uint64_t sv[3] = {(uint64_t)(st[8] * 4), (uint64_t)(st[7] * 4), (uint64_t)(st[6] * 4)};
    if (int rc = make_tmap(&tv, v, 4, dims, sv, box, 4, /*atom32=*/true)) return rc;
  }
  SdpaArgs a{};
  a.B = (int)B;
  a.T = (int)T;
  a.S = (int)S;
  a.N = (int)N;
  a.scale = scale;
  a.causal = causal;
  a.o = o;
  a.o_sb = st[9];
  a.o_st = st[10];
  a.o_sn = st[11];
  a.err = device_error_word();
  if (!a.err) return set_error(B200_ERR_CUDA, "could not allocate the device error word");
  if (int rc = allow_dynamic_smem((const void*)sdpa_fwd_tc_x3, X3Cfg::SMEM, "sdpa_fwd_tc_x3")) return rc;
  dim3 grid((unsigned)((T + 127) / 128), (unsigned)N, (unsigned)B);
  B200_LAUNCH(sdpa_fwd_tc_x3, grid, dim3(128), X3Cfg::SMEM, s, tq, tk, tv, a);
  return B200_OK;
}

// ---------------------------------------------------------------------------
// Attention backward, bf16, head dim 64, T == S <= 256 (flash-style: P is
// recomputed from the forward's row statistics, the [T, S] matrices never
// touch HBM).
//
// One CTA = one (batch, head); Q, dO, K and V (at most 2 tiles of 128 rows
// each) are loaded once by TMA and stay in shared memory.  Query tile i and
// key tile j form a pair (j outer; causal: i >= j).  17 warps (544 threads):
//   warps 0-15 warp w reads TMEM lane quarter w % 4 (32 query rows) and key
//     columns 32 (w / 4) .. +31 of S and dP, forms P = 2^(S*scale*log2e -
//     lse2) and dS = P (dP - D) scale in f32, with D = rowsum(dO * O), and
//     writes P as bf16 (the precision jax.nn.dot_product_attention gives the
//     probabilities) and dS as bf16 hi + lo (about 16 significant bits, like
//     the f32 dS of the unfused program) into shared memory (two 64-key chunks
//     of 128-byte rows, 16-byte units XOR row % 8); after the last pair of key
//     tile j the warps store dK_j and dV_j, and at the end every dQ_i;
//   warp 16   lane 0 issues the TMA loads and the MMAs: S = Q_i K_j^T
//     and dP = dO_i V_j^T (M = N = 128) into TMEM, and once P / dS are in
//     shared memory dV_j += P^T dO_i, dK_j += dS^T Q_i (A operands MN-major)
//     and dQ_i += dS K_j (B MN-major), each dS product as two MMAs (hi, lo).
//     The next pair's S / dP are issued as soon as every warp holds the
//     current ones in registers, so the tensor core runs them and the
//     previous pair's dV / dK / dQ while the warps compute (issuing blocks
//     while the tensor core's queue is full, so it has a warp of its own).
// D is formed first with coalesced loads of O and dO (8 lanes per 128-byte
// row) and kept in shared memory.  dK_j / dV_j go out through the K_j / V_j
// tiles (free once key tile j is done) and dQ_i through Q_i, as TMA stores.
// TMEM columns: S 0-127, dP 128-255, dV 256-319, dK 320-383, dQ_i 384 + 64 i.
// Math: the vjp of softmax(QK^T*scale)V (reference src/jax_mlx/sdpa.py:65-87,
// whose mlx_sdpa_bwd the reference runs through mx::vjp,
// src/jax_mlx_pjrt.cpp:8152-8206).
struct BwdArgs {
  int B, T, N;
  float scale;
  int causal;
  const float* lse2;  // [B, N, T]: log2 of each row's sum_s 2^(scale*log2(e)*q.k_s)
  const __nv_bfloat16* o;
  int64_t o_sb, o_st, o_sn;
  const __nv_bfloat16* dout;
  int64_t do_sb, do_st, do_sn;
  __nv_bfloat16* dq;
  int64_t dq_sb, dq_st, dq_sn;
  __nv_bfloat16* dk;
  int64_t dk_sb, dk_st, dk_sn;
  __nv_bfloat16* dv;
  int64_t dv_sb, dv_st, dv_sn;
  int* err;
};

struct BwdCfg {
  static constexpr int TILE = 128 * 128;  // 128 rows x 128 B (64 bf16)
  static constexpr int Q_OFF = 0;         // 2 tiles each
  static constexpr int DO_OFF = Q_OFF + 2 * TILE;
  static constexpr int K_OFF = DO_OFF + 2 * TILE;
  static constexpr int V_OFF = K_OFF + 2 * TILE;
  static constexpr int P_OFF = V_OFF + 2 * TILE;     // 2 chunks of 64 keys
  static constexpr int DS_OFF = P_OFF + 2 * TILE;    // dS as bf16 hi ...
  static constexpr int DSL_OFF = DS_OFF + 2 * TILE;  // ... and lo (rounded residual)
  static constexpr int D_OFF = DSL_OFF + 2 * TILE;  // D per query row (f32, 2 tiles)
  static constexpr int BAR_OFF = D_OFF + 2 * 128 * 4;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
  static_assert(SMEM <= 232448, "shared memory above the 227 KB per-block limit");
};
constexpr int kBwdWarps = 16;                       // compute warps
constexpr int kBwdThreads = (kBwdWarps + 1) * 32;  // + the issue warp

__global__ void __launch_bounds__(kBwdThreads, 1)
    sdpa_bwd_tc(const __grid_constant__ CUtensorMap tQ, const __grid_constant__ CUtensorMap tK,
                const __grid_constant__ CUtensorMap tV, const __grid_constant__ CUtensorMap tDO,
                const __grid_constant__ CUtensorMap mDQ, const __grid_constant__ CUtensorMap mDK,
                const __grid_constant__ CUtensorMap mDV, BwdArgs p) {
  pdl_wait();
  using C = BwdCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* ld_full = bars + 0;   // every Q / dO / K / V tile landed
  uint64_t* sd_full = bars + 1;   // S and dP of a pair in TMEM (one phase per pair)
  uint64_t* s_free = bars + 2;    // S and dP read into registers (16 warps)
  uint64_t* pds_full = bars + 3;  // P and dS in shared memory (16 warps)
  uint64_t* acc_done = bars + 4;  // the pair's dV / dK / dQ MMAs complete
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool issuer = tid == kBwdWarps * 32;
  const int n = (int)blockIdx.x % p.N, b = (int)blockIdx.x / p.N;
  const int nt = (p.T + 127) / 128;
  auto tile = [&](int off, int i) { return smem + off + i * C::TILE; };
  // the pairs in order: key tile j outer, query tile i inner (causal: i >= j)
  const int np = p.causal ? nt * (nt + 1) / 2 : nt * nt;
  auto pair_i = [&](int k) {
    if (!p.causal) return k % nt;
    for (int j = 0; j < nt; ++j) {
      if (k < nt - j) return j + k;
      k -= nt - j;
    }
    return 0;
  };
  auto pair_j = [&](int k) {
    if (!p.causal) return k / nt;
    for (int j = 0; j < nt; ++j) {
      if (k < nt - j) return j;
      k -= nt - j;
    }
    return 0;
  };

  if (issuer) {
    mbar_init(ld_full, 1);
    mbar_init(sd_full, 1);
    mbar_init(s_free, kBwdWarps);
    mbar_init(pds_full, kBwdWarps);
    mbar_init(acc_done, 1);
    *abort = 0;
    mbar_fence_init();
  }
  if (warp == kBwdWarps) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tS = tmem, tDP = tmem + 128u, tDV = tmem + 256u, tDK = tmem + 320u;

  // ---- MMA issue (thread 0)
  constexpr uint32_t idesc_s = umma_idesc(1u, 0, 0, 128, 128);  // K-major x K-major
  constexpr uint32_t idesc_t = umma_idesc(1u, 1, 1, 64, 128);   // P^T / dS^T times dO / Q
  constexpr uint32_t idesc_q = umma_idesc(1u, 0, 1, 64, 128);   // dS times K
  auto issue_sd = [&](int k) {  // S and dP of pair k
    const uint32_t qt = smem_u32(tile(C::Q_OFF, pair_i(k))), dot = smem_u32(tile(C::DO_OFF, pair_i(k)));
    const uint32_t kt = smem_u32(tile(C::K_OFF, pair_j(k))), vt = smem_u32(tile(C::V_OFF, pair_j(k)));
    tc_fence_after();
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      umma_f16(tS, umma_desc(qt + kk * 32, 16, 1024), umma_desc(kt + kk * 32, 16, 1024), idesc_s, kk != 0);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      umma_f16(tDP, umma_desc(dot + kk * 32, 16, 1024), umma_desc(vt + kk * 32, 16, 1024), idesc_s, kk != 0);
    umma_commit(sd_full);
  };
  auto issue_acc = [&](int k) {  // dV, dK, dQ of pair k
    const int i = pair_i(k), j = pair_j(k);
    const int i0 = p.causal ? j : 0;
    const uint32_t pp = smem_u32(smem + C::P_OFF), ds = smem_u32(smem + C::DS_OFF);
    const uint32_t dsl = smem_u32(smem + C::DSL_OFF);
    const uint32_t qt = smem_u32(tile(C::Q_OFF, i)), dot = smem_u32(tile(C::DO_OFF, i));
    const uint32_t kt = smem_u32(tile(C::K_OFF, j));
    const uint32_t tDQ = tmem + 384u + 64u * (uint32_t)i;
    // descriptors are built once; a byte offset moves the start address field
    // (bits 0-13, in 16-byte units)
    const uint64_t dP = umma_desc(pp, 16384, 1024), dDS = umma_desc(ds, 16384, 1024);
    const uint64_t dDSL = umma_desc(dsl, 16384, 1024), dDO = umma_desc(dot, 8192, 1024);
    const uint64_t dQt = umma_desc(qt, 8192, 1024), dKt = umma_desc(kt, 8192, 1024);
    const uint64_t dDSk = umma_desc(ds, 16, 1024), dDSLk = umma_desc(dsl, 16, 1024);
    tc_fence_after();
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      // 16 queries = 16 rows of 128 B in P / dS (MN-major A: the two 64-key
      // chunks 16 KB apart) and in dO / Q (MN-major B)
      const uint32_t ka = (uint32_t)(i != i0 || kk != 0);
      const uint64_t o16 = (uint64_t)(kk * 2048 >> 4);
      umma_f16(tDV, dP + o16, dDO + o16, idesc_t, ka);
      umma_f16(tDK, dDS + o16, dQt + o16, idesc_t, ka);
      umma_f16(tDK, dDSL + o16, dQt + o16, idesc_t, 1);
      // 16 keys: 32 bytes of a dS row (K-major A), 16 rows of K (MN-major B)
      const uint64_t a16 = (uint64_t)(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
      umma_f16(tDQ, dDSk + a16, dKt + o16, idesc_q, (uint32_t)(j != 0 || kk != 0));
      umma_f16(tDQ, dDSLk + a16, dKt + o16, idesc_q, 1);
    }
    umma_commit(acc_done);
  };
  if (issuer) {
    tma_prefetch_desc(&tQ);
    tma_prefetch_desc(&tK);
    tma_prefetch_desc(&tV);
    tma_prefetch_desc(&tDO);
    tma_prefetch_desc(&mDQ);
    tma_prefetch_desc(&mDK);
    tma_prefetch_desc(&mDV);
    mbar_expect_tx(ld_full, 4 * nt * C::TILE);
    for (int i = 0; i < nt; ++i) {
      tma_load_4d(tile(C::Q_OFF, i), &tQ, ld_full, 0, n, i * 128, b);
      tma_load_4d(tile(C::DO_OFF, i), &tDO, ld_full, 0, n, i * 128, b);
      tma_load_4d(tile(C::K_OFF, i), &tK, ld_full, 0, n, i * 128, b);
      tma_load_4d(tile(C::V_OFF, i), &tV, ld_full, 0, n, i * 128, b);
    }
  }

  // ---- D = rowsum(dO * O) per query row (while the tiles load): a compute
  // warp takes 8 rows per tile, 8 lanes per 128-byte row
  float* dsm = reinterpret_cast<float*>(smem + C::D_OFF);
  if (warp < kBwdWarps) {
    for (int i = 0; i < nt; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = warp * 8 + h * 4 + (lane >> 3), t = i * 128 + row;
        float acc = 0.f;
        if (t < p.T) {
          const uint4 x = reinterpret_cast<const uint4*>(p.o + (int64_t)b * p.o_sb + (int64_t)t * p.o_st +
                                                         (int64_t)n * p.o_sn)[lane & 7];
          const uint4 y = reinterpret_cast<const uint4*>(p.dout + (int64_t)b * p.do_sb + (int64_t)t * p.do_st +
                                                         (int64_t)n * p.do_sn)[lane & 7];
          const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xs[c]));
            const float2 g = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ys[c]));
            acc = fmaf(a.x, g.x, fmaf(a.y, g.y, acc));
          }
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        acc += __shfl_xor_sync(0xffffffffu, acc, 4);
        if ((lane & 7) == 0) dsm[i * 128 + row] = acc;
      }
  }
  __syncthreads();
  const int qq = warp & 3, cg = warp >> 2;
  const int r = qq * 32 + lane;  // row within a 128-row tile (= TMEM lane)
  const uint32_t lane_base = (uint32_t)(qq * 32) << 16;
  const float sl2 = p.scale * 1.4426950408889634f;
  float lse0 = 0.f, lse1 = 0.f, d0 = 0.f, d1 = 0.f;
  for (int i = 0; i < nt; ++i) {
    const int t = i * 128 + r;
    if (t >= p.T) continue;
    const float l = p.lse2[((int64_t)b * p.N + n) * p.T + t];
    if (i == 0) { lse0 = l; d0 = dsm[r]; } else { lse1 = l; d1 = dsm[128 + r]; }
  }
  if (warp == kBwdWarps) {
    if (issuer) {  // ---- MMA issue
      bool ok = mbar_wait(ld_full, 0, abort, p.err, 231);
      if (ok) issue_sd(0);
      for (int k = 0; ok && k < np; ++k) {
        ok = mbar_wait(s_free, k & 1, abort, p.err, 232);
        if (!ok) break;
        if (k + 1 < np) issue_sd(k + 1);  // the S / dP buffers are free again
        ok = mbar_wait(pds_full, k & 1, abort, p.err, 236);
        if (ok) issue_acc(k);
      }
    }
  } else {  // ---- warps 0-15
    // A 128 x 64 f32 accumulator (TMEM columns `tcol`) -> bf16 tile in
    // shared memory (128-byte rows, 16-byte units XOR row % 8, the TMA
    // layout): this warp's lane quarter, columns 16 cg .. +15
    auto stage = [&](uint32_t tcol, uint8_t* dst) {
      float v[16];
      tmem_ld16(tcol + lane_base + (uint32_t)(cg * 16), v);
#pragma unroll
      for (int u = 0; u < 2; ++u)
        *reinterpret_cast<uint4*>(dst + r * 128 + (((cg * 2 + u) ^ (r & 7)) << 4)) =
            make_uint4(pack_bf16x2(v[8 * u], v[8 * u + 1]), pack_bf16x2(v[8 * u + 2], v[8 * u + 3]),
                       pack_bf16x2(v[8 * u + 4], v[8 * u + 5]), pack_bf16x2(v[8 * u + 6], v[8 * u + 7]));
    };
    // dK_j and dV_j once the last pair of key tile j has completed (rows are
    // keys), staged in the K_j / V_j tiles and written by one TMA store each
    auto store_kv = [&](int j) {
      stage(tDV, tile(C::V_OFF, j));
      stage(tDK, tile(C::K_OFF, j));
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, %0;" ::"n"(kBwdWarps * 32) : "memory");
      if (tid == 0) {
        tma_store_4d(&mDV, tile(C::V_OFF, j), 0, n, j * 128, b);
        tma_store_4d(&mDK, tile(C::K_OFF, j), 0, n, j * 128, b);
        bulk_commit_group();
      }
    };
    const int col = cg * 32;  // this warp's key columns within a tile
    uint8_t* prow = smem + C::P_OFF + (cg >> 1) * C::TILE + r * 128;
    uint8_t* drow = smem + C::DS_OFF + (cg >> 1) * C::TILE + r * 128;
    uint8_t* lrow = smem + C::DSL_OFF + (cg >> 1) * C::TILE + r * 128;
    bool ok = true;
    for (int k = 0; k < np; ++k) {
      const int i = pair_i(k), j = pair_j(k);
      bool w = mbar_wait(sd_full, k & 1, abort, p.err, 233);
      if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[32], dr[32];
      tmem_ld32_async(tS + lane_base + (uint32_t)col, sr);
      tmem_ld32_async(tDP + lane_base + (uint32_t)col, dr);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);  // the next pair's S / dP may overwrite TMEM now
      const int t = i * 128 + r;
      const bool row_ok = t < p.T;
      const float li = i ? lse1 : lse0, di = i ? d1 : d0;
      const int kb = j * 128 + col;
      // keys up to `lim` count: below T, at or before the query when causal,
      // none for a padding row (one compare per element)
      const int lim = !row_ok ? -1 : p.causal ? min(t, p.T - 1) : p.T - 1;
      uint32_t pw[16], dw[16], dl[16];
#pragma unroll
      for (int x = 0; x < 16; ++x) {
        float pv[2], dv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kb + 2 * x + e;
          const bool valid = key <= lim;
          pv[e] = valid ? ex2(fmaf(__uint_as_float(sr[2 * x + e]), sl2, -li)) : 0.f;
          dv[e] = pv[e] * (__uint_as_float(dr[2 * x + e]) - di) * p.scale;
        }
        pw[x] = pack_bf16x2(pv[0], pv[1]);
        __nv_bfloat162 hh = __floats2bfloat162_rn(dv[0], dv[1]);
        dw[x] = *reinterpret_cast<uint32_t*>(&hh);
        const float2 hf = __bfloat1622float2(hh);
        dl[x] = pack_bf16x2(dv[0] - hf.x, dv[1] - hf.y);
      }
      // P / dS of the previous pair are read by its MMAs until acc_done; a key
      // tile finished by that pair is stored before the next MMAs reuse its
      // accumulators
      if (k > 0) {
        w = mbar_wait(acc_done, (k - 1) & 1, abort, p.err, 234);
        if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
        tc_fence_after();
        if (pair_j(k - 1) != j) store_kv(pair_j(k - 1));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int off = (((cg & 1) * 4 + u) ^ (r & 7)) << 4;
        *reinterpret_cast<uint4*>(prow + off) = make_uint4(pw[4 * u], pw[4 * u + 1], pw[4 * u + 2], pw[4 * u + 3]);
        *reinterpret_cast<uint4*>(drow + off) = make_uint4(dw[4 * u], dw[4 * u + 1], dw[4 * u + 2], dw[4 * u + 3]);
        *reinterpret_cast<uint4*>(lrow + off) = make_uint4(dl[4 * u], dl[4 * u + 1], dl[4 * u + 2], dl[4 * u + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pds_full);
    }
    if (ok) {
      const bool w = mbar_wait(acc_done, (np - 1) & 1, abort, p.err, 235);
      ok = __all_sync(0xffffffffu, w) != 0;
    }
    if (ok) {  // every MMA has completed
      tc_fence_after();
      store_kv(pair_j(np - 1));
      // dQ_i staged in the Q_i tiles (no MMA reads them any more)
      for (int i = 0; i < nt; ++i) stage(tmem + 384u + 64u * (uint32_t)i, tile(C::Q_OFF, i));
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, %0;" ::"n"(kBwdWarps * 32) : "memory");
      if (tid == 0) {
        for (int i = 0; i < nt; ++i) tma_store_4d(&mDQ, tile(C::Q_OFF, i), 0, n, i * 128, b);
        bulk_commit_group();
      }
    }
    if (tid == 0) bulk_wait_group_read<0>();  // shared memory stays valid until read
  }
  tc_fence_before();
  __syncthreads();
  if (*abort && tid == 0) {  // let MMAs still in flight drain before TMEM is freed
    const uint64_t t1 = globaltimer();
    while (globaltimer() - t1 < 2000000ull) {
    }
  }
  __syncthreads();
  if (warp == kBwdWarps) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int launch_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
               const float* lse2, void* dq, void* dk, void* dv, int64_t B, int64_t T, int64_t N,
               const int64_t* st, float scale, int causal, cudaStream_t s) {
  // st: (b, t, n) element strides of q, k, v, o, dout, dq, dk, dv
  CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
  const void* src[7] = {q, k, v, dout, dq, dk, dv};
  const int sidx[7] = {0, 1, 2, 4, 5, 6, 7};
  CUtensorMap* maps[7] = {&tq, &tk, &tv, &tdo, &tdq, &tdk, &tdv};
  for (int m = 0; m < 7; ++m) {
    const int64_t* x = st + 3 * sidx[m];
    const uint64_t dims[4] = {64, (uint64_t)N, (uint64_t)T, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)(x[2] * 2), (uint64_t)(x[1] * 2), (uint64_t)(x[0] * 2)};
    const uint32_t box[4] = {64, 1, 128, 1};
    if (int rc = make_tmap(maps[m], src[m], 4, dims, str, box, 2)) return rc;
  }
  BwdArgs a{};
  a.B = (int)B;
  a.T = (int)T;
  a.N = (int)N;
  a.scale = scale;
  a.causal = causal;
  a.lse2 = lse2;
  a.o = (const __nv_bfloat16*)o;
  a.o_sb = st[9], a.o_st = st[10], a.o_sn = st[11];
  a.dout = (const __nv_bfloat16*)dout;
  a.do_sb = st[12], a.do_st = st[13], a.do_sn = st[14];
  a.dq = (__nv_bfloat16*)dq;
  a.dq_sb = st[15], a.dq_st = st[16], a.dq_sn = st[17];
  a.dk = (__nv_bfloat16*)dk;
  a.dk_sb = st[18], a.dk_st = st[19], a.dk_sn = st[20];
  a.dv = (__nv_bfloat16*)dv;
  a.dv_sb = st[21], a.dv_st = st[22], a.dv_sn = st[23];
  a.err = device_error_word();
  if (!a.err) return set_error(B200_ERR_CUDA, "could not allocate the device error word");
  if (int rc = allow_dynamic_smem((const void*)sdpa_bwd_tc, BwdCfg::SMEM, "sdpa_bwd_tc")) return rc;
  B200_LAUNCH(sdpa_bwd_tc, dim3((unsigned)(B * N)), dim3(kBwdThreads), BwdCfg::SMEM, s, tq, tk, tv,
              tdo, tdq, tdk, tdv, a);
  return B200_OK;
}

}  // namespace
}  // namespace b200

extern "C" int b200_sdpa_fwd_strided(const void* q, const void* k, const void* v, void* o,
                                     int64_t B, int64_t T, int64_t S, int64_t N, int64_t D,
                                     const int64_t* st, float scale, int causal, int dtype,
                                     void* stream) {
  using namespace b200;
  B200_CHECK_ARG(q && k && v && o && st, "sdpa: null argument");
  B200_CHECK_ARG(B > 0 && T > 0 && S > 0 && N > 0 && D > 0, "sdpa: bad shape");
  B200_CHECK_ARG(B < 65536 && N < 65536 && T < (1 << 30) && S < (1 << 30), "sdpa: shape too large");
  B200_CHECK_ARG(dtype == B200_DT_F32 || dtype == B200_DT_BF16, "sdpa: dtype must be F32 or BF16");
  auto s = (cudaStream_t)stream;
  const int es = dtype == B200_DT_F32 ? 4 : 2;
  bool tc = D == 64;
  for (int i = 0; i < 12; ++i) tc = tc && ((st[i] * es) % 16 == 0);
  const void* ptrs[4] = {q, k, v, o};
  for (int i = 0; i < 4; ++i) tc = tc && ((uintptr_t)ptrs[i] % 16 == 0);
  if (tc) {
    static const bool legacy = [] {
      const char* e = std::getenv("B200_SDPA_LEGACY");
      return e && std::strcmp(e, "1") == 0;
    }();
    if (!legacy && scale > 0.f) {  // (the kernel masks with -inf before scaling)
      if (es == 4) return launch_ws<true>(q, k, v, o, B, T, S, N, st, scale, causal, s);
      return launch_ws<false>(q, k, v, o, B, T, S, N, st, scale, causal, s);
    }
    if (es == 4) {
      static const bool x3 = [] {
        const char* e = std::getenv("B200_F32_MATMUL");
        return !(e && std::strcmp(e, "tf32") == 0);
      }();
      if (x3) return launch_x3(q, k, v, o, B, T, S, N, st, scale, causal, s);
      return launch_tc<4>(q, k, v, o, B, T, S, N, st, scale, causal, s);
    }
    return launch_tc<2>(q, k, v, o, B, T, S, N, st, scale, causal, s);
  }
  B200_CHECK_ARG(S <= 8192, "sdpa: the fallback kernel supports S <= 8192");
  // strides to device memory (small, stream-ordered)
  int64_t* dst = nullptr;
  B200_CUDA_TRY(cudaMallocAsync((void**)&dst, 12 * sizeof(int64_t), s));
  B200_CUDA_TRY(cudaMemcpyAsync(dst, st, 12 * sizeof(int64_t), cudaMemcpyHostToDevice, s));
  const size_t smem = (size_t)(S + D) * sizeof(float);
  dim3 grid((unsigned)T, (unsigned)N, (unsigned)B);
  if (es == 4)
    B200_LAUNCH(sdpa_fwd_simt<float>, grid, dim3(128), smem, s, (const float*)q, (const float*)k,
                (const float*)v, (float*)o, (int)S, (int)D, (const int64_t*)dst, scale, causal);
  else
    B200_LAUNCH(sdpa_fwd_simt<__nv_bfloat16>, grid, dim3(128), smem, s, (const __nv_bfloat16*)q,
                (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (__nv_bfloat16*)o, (int)S, (int)D,
                (const int64_t*)dst, scale, causal);
  B200_CUDA_TRY(cudaFreeAsync(dst, s));
  return B200_OK;
}

extern "C" int b200_sdpa_fwd(const void* q, const void* k, const void* v, void* o, int64_t B,
                             int64_t T, int64_t S, int64_t N, int64_t D, float scale, int causal,
                             int dtype, void* stream) {
  const int64_t st[12] = {T * N * D, N * D, D, S * N * D, N * D, D,
                          S * N * D, N * D, D, T * N * D, N * D, D};
  return b200_sdpa_fwd_strided(q, k, v, o, B, T, S, N, D, st, scale, causal, dtype, stream);
}

extern "C" int b200_sdpa_fwd_lse(const void* q, const void* k, const void* v, void* o, float* lse2,
                                 int64_t B, int64_t T, int64_t S, int64_t N, int64_t D,
                                 const int64_t* st, float scale, int causal, int dtype,
                                 void* stream) {
  using namespace b200;
  B200_CHECK_ARG(q && k && v && o && lse2 && st, "sdpa_fwd_lse: null argument");
  B200_CHECK_ARG(B > 0 && T > 0 && S > 0 && N > 0 && D > 0, "sdpa_fwd_lse: bad shape");
  B200_CHECK_ARG(B < 65536 && N < 65536 && T < (1 << 30) && S < (1 << 30),
                 "sdpa_fwd_lse: shape too large");
  B200_CHECK_ARG(dtype == B200_DT_F32 || dtype == B200_DT_BF16,
                 "sdpa_fwd_lse: dtype must be F32 or BF16");
  const int es = dtype == B200_DT_F32 ? 4 : 2;
  bool tc = D == 64 && scale > 0.f;
  for (int i = 0; i < 12; ++i) tc = tc && ((st[i] * es) % 16 == 0);
  const void* ptrs[4] = {q, k, v, o};
  for (int i = 0; i < 4; ++i) tc = tc && ((uintptr_t)ptrs[i] % 16 == 0);
  if (!tc)
    return set_error(B200_ERR_UNSUPPORTED,
                     "sdpa_fwd_lse: needs D == 64, scale > 0 and 16-byte aligned operands and strides");
  auto s = (cudaStream_t)stream;
  if (es == 4) return launch_ws<true>(q, k, v, o, B, T, S, N, st, scale, causal, s, lse2);
  return launch_ws<false>(q, k, v, o, B, T, S, N, st, scale, causal, s, lse2);
}

extern "C" int b200_sdpa_bwd(const void* q, const void* k, const void* v, const void* o,
                             const void* dout, const float* lse2, void* dq, void* dk, void* dv,
                             int64_t B, int64_t T, int64_t N, int64_t D, const int64_t* st,
                             float scale, int causal, int dtype, void* stream) {
  using namespace b200;
  B200_CHECK_ARG(q && k && v && o && dout && lse2 && dq && dk && dv && st, "sdpa_bwd: null argument");
  B200_CHECK_ARG(B > 0 && T > 0 && N > 0 && D > 0, "sdpa_bwd: bad shape");
  B200_CHECK_ARG((int64_t)B * N < (1ll << 31), "sdpa_bwd: too many (batch, head) pairs");
  if (dtype != B200_DT_BF16 || D != 64 || T > 256)
    return set_error(B200_ERR_UNSUPPORTED, "sdpa_bwd: needs bf16, head dim 64 and T <= 256");
  bool al = true;
  for (int i = 0; i < 24; ++i) al = al && (st[i] % 8 == 0);
  const void* ptrs[8] = {q, k, v, o, dout, dq, dk, dv};
  for (int i = 0; i < 8; ++i) al = al && ((uintptr_t)ptrs[i] % 16 == 0);
  if (!al) return set_error(B200_ERR_UNSUPPORTED, "sdpa_bwd: operands and strides must be 16-byte aligned");
  return launch_bwd(q, k, v, o, dout, lse2, dq, dk, dv, B, T, N, st, scale, causal,
                    (cudaStream_t)stream);
}
