// Batched GEMM for dot_general and convolution (im2col) on sm_100a.
//
// Tensor-core path: one 128 x BN output tile per CTA, 192 threads in three
// roles -- warp 0 issues TMA loads into a 4-stage shared-memory ring, warp 1
// issues tcgen05.mma (kind::tf32 for f32 operands, kind::f16 for bf16) into a
// TMEM accumulator, warps 2-5 drain TMEM (tcgen05.ld) through the epilogue
// (alpha, bias, ReLU, f32/bf16 store).  Operands may be K-major or MN-major
// (transposed) views: the TMA descriptor and the UMMA descriptor's majorness
// absorb the transpose, so no copy is made.  Shapes or strides TMA cannot
// express (rows not 16-byte aligned, e.g. N = 10 in f32) use a SIMT kernel
// with f32 FMAs.
//
// Replaces reference src/jax_mlx_pjrt.cpp:4577-4666 (dot_general lowered to
// transpose + reshape + mlx::core::matmul).
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "gemm_ws.h"
#include "tc.cuh"

namespace b200 {
namespace {


struct GemmArgs {
  int M, N, K;
  int a_mn, b_mn;
  float alpha;
  const void* bias;
  int epi;  // 0 none, 1 bias, 2 bias+relu, 3 relu
  void* c;
  int64_t ldc, sCb;
  int* err;
  // split-K: gridDim.z = batch * splits; split s covers k-blocks
  // [s*kb_per_split, (s+1)*kb_per_split) and writes raw f32 partial sums to
  // ws[(b*splits + s)][M][N] (alpha/bias/activation applied by splitk_reduce).
  int splits, kb_per_split;
  float* ws;
};

template <typename TO>
__device__ __forceinline__ void store_out(TO* p, float v);
template <>
__device__ __forceinline__ void store_out<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store_out<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}
template <typename TO>
__device__ __forceinline__ float load_bias(const void* b, int n) {
  return Io<TO>::to_f(reinterpret_cast<const TO*>(b)[n]);
}

// Stage count and shared-memory bytes of one gemm_tc configuration.
template <int BN, int ES, bool SPLIT>
struct TcCfg {
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE = (A_BYTES + B_BYTES) * (SPLIT ? 2 : 1);
  static constexpr int STAGES = (STAGE * 4 <= 200 * 1024) ? 4 : 3;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
};

// f32 -> tf32 with round-to-nearest (ties away); low 13 mantissa bits cleared.
__device__ __forceinline__ float to_tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi/lo split of a staged f32 tile in place: tile <- tf32(x), lo <- x - tf32(x).
// Elementwise, so the TMA's swizzled layout carries over to both copies.
__device__ __forceinline__ void split_tile(uint8_t* tile, uint8_t* lo, int bytes, int tid, int nthr) {
  for (int off = tid * 16; off < bytes; off += nthr * 16) {
    float4 v = *reinterpret_cast<float4*>(tile + off);
    float4 h = make_float4(to_tf32_rna(v.x), to_tf32_rna(v.y), to_tf32_rna(v.z), to_tf32_rna(v.w));
    *reinterpret_cast<float4*>(tile + off) = h;
    *reinterpret_cast<float4*>(lo + off) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
  }
}

// SPLIT (f32 operands only): 3xTF32 -- each operand is split into tf32 hi and
// lo parts in shared memory by warps 2-5 and the MMA warp accumulates
// A_lo*B_hi + A_hi*B_lo + A_hi*B_hi, which keeps f32-level accuracy (the
// dropped A_lo*B_lo term is below 2^-20 relative).
template <int BN, int ES, typename TO, bool SPLIT>
__global__ void __launch_bounds__(192, 1)
    gemm_tc(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
            GemmArgs p) {
  pdl_wait();
  using Cfg = TcCfg<BN, ES, SPLIT>;
  constexpr int S = Cfg::STAGES;
  constexpr int BK = 128 / ES;  // K elements per 128-byte row
  constexpr int E = 128 / ES;   // MN elements per 128-byte chunk
  constexpr int A_BYTES = Cfg::A_BYTES;
  constexpr int B_BYTES = Cfg::B_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  // stage s: [A | B | A_lo | B_lo]
  auto sA = [&](int s) { return smem + s * Cfg::STAGE; };
  auto sB = [&](int s) { return smem + s * Cfg::STAGE + A_BYTES; };
  auto sAlo = [&](int s) { return smem + s * Cfg::STAGE + A_BYTES + B_BYTES; };
  auto sBlo = [&](int s) { return smem + s * Cfg::STAGE + 2 * A_BYTES + B_BYTES; };
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::STAGE);
  uint64_t* split = full + S;
  uint64_t* empty = split + S;
  uint64_t* tfull = empty + S;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tfull + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * 128;
  const int bz = blockIdx.z / p.splits, ks = blockIdx.z % p.splits;
  const int KB_all = (p.K + BK - 1) / BK;
  const int kb0 = ks * p.kb_per_split;
  const int KB = max(0, min(KB_all, kb0 + p.kb_per_split) - kb0);  // k-blocks of this CTA

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&split[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    *abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tA);
    tma_prefetch_desc(&tB);
  }
  if (warp == 0) {
    tmem_alloc(tslot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      for (int i = 0; i < KB; ++i) {
        const int s = i % S, kb = kb0 + i;
        if (i >= S && !mbar_wait(&empty[s], ((i / S) + 1) & 1, abort, p.err, 101)) break;
        mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
        if (!p.a_mn) {
          tma_load_3d(sA(s), &tA, &full[s], kb * BK, m0, bz);
        } else {
#pragma unroll
          for (int i = 0; i < 128 / E; ++i)
            tma_load_3d(sA(s) + i * (BK * 128), &tA, &full[s], m0 + i * E, kb * BK, bz);
        }
        if (!p.b_mn) {
          tma_load_3d(sB(s), &tB, &full[s], kb * BK, n0, bz);
        } else {
#pragma unroll
          for (int i = 0; i < BN / E; ++i)
            tma_load_3d(sB(s) + i * (BK * 128), &tB, &full[s], n0 + i * E, kb * BK, bz);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = umma_idesc(ES == 4 ? 2u : 1u, (uint32_t)p.a_mn, (uint32_t)p.b_mn, BN, 128);
      constexpr uint32_t KSTEP_MN = (32 / ES) * 128;  // bytes per MMA K-step, MN-major
      constexpr uint32_t MN_LAYOUT = ES == 4 ? kUmmaSW128Base32 : kUmmaSW128;
      constexpr uint32_t MN_SBO = ES == 4 ? 512 : 1024;
      // MN-major: LBO = stride between 128-byte MN chunks (one TMA box each),
      // SBO = stride between K-row groups (8 rows of 128 B; 4 for the tf32 layout)
      auto adesc = [&](uint32_t base, int kk) {
        return p.a_mn ? umma_desc(base + kk * KSTEP_MN, BK * 128, MN_SBO, MN_LAYOUT)
                      : umma_desc(base + kk * 32, 16, 1024);
      };
      auto bdesc = [&](uint32_t base, int kk) {
        return p.b_mn ? umma_desc(base + kk * KSTEP_MN, BK * 128, MN_SBO, MN_LAYOUT)
                      : umma_desc(base + kk * 32, 16, 1024);
      };
      bool ok = true;
      for (int i = 0; i < KB; ++i) {
        const int s = i % S;
        const bool w = SPLIT ? mbar_wait(&split[s], (i / S) & 1, abort, p.err, 102)
                             : mbar_wait(&full[s], (i / S) & 1, abort, p.err, 102);
        if (!w) { ok = false; break; }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA(s)), b0 = smem_u32(sB(s));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = adesc(a0, kk), bd = bdesc(b0, kk);
          if (ES == 4) {
            if (SPLIT) {
              umma_tf32(tmem, adesc(smem_u32(sAlo(s)), kk), bd, idesc, (i | kk) != 0);
              umma_tf32(tmem, ad, bdesc(smem_u32(sBlo(s)), kk), idesc, 1);
              umma_tf32(tmem, ad, bd, idesc, 1);
            } else {
              umma_tf32(tmem, ad, bd, idesc, (i | kk) != 0);
            }
          } else {
            umma_f16(tmem, ad, bd, idesc, (i | kk) != 0);
          }
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(tfull);
    }
  } else {  // ---- warps 2..5: operand split (3xTF32), then the epilogue
    if (SPLIT) {
      const int tid = threadIdx.x - 64;
      for (int i = 0; i < KB; ++i) {
        const int s = i % S;
        bool w = mbar_wait(&full[s], (i / S) & 1, abort, p.err, 104);
        if (!__all_sync(0xffffffffu, w)) break;
        split_tile(sA(s), sAlo(s), A_BYTES, tid, 128);
        split_tile(sB(s), sBlo(s), B_BYTES, tid, 128);
        fence_proxy_async_smem();  // generic-proxy writes -> visible to tcgen05.mma
        __syncwarp();
        if (lane == 0) mbar_arrive(&split[s]);
      }
    }
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int m = m0 + row;
    bool ok = KB == 0 || mbar_wait(tfull, 0, abort, p.err, 103);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (ok && p.splits > 1) {
      float* prow = p.ws + ((int64_t)blockIdx.z * p.M + m) * p.N;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        if (KB > 0) {
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        if (m < p.M) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + c + j < p.N) prow[n0 + c + j] = v[j];
        }
      }
    } else if (ok) {
      TO* crow = reinterpret_cast<TO*>(p.c) + (int64_t)bz * p.sCb + (int64_t)m * p.ldc;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
        if (m < p.M) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = n0 + c + j;
            if (n < p.N) {
              float x = v[j] * p.alpha;
              if (p.epi == 1 || p.epi == 2) x += load_bias<TO>(p.bias, n);
              if (p.epi >= 2) x = fmaxf(x, 0.f);
              store_out<TO>(crow + n, x);
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort && threadIdx.x == 0) {
    // let TMA copies already in flight land before the CTA's shared memory goes away
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 2000000ull) {
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

// ---------------------------------------------------------------------------
// Persistent bf16 GEMM: one CTA per SM walks a static tile schedule
// (t = blockIdx.x, += gridDim.x).  Warp 0 streams A/B k-blocks through an
// S-stage TMA ring that runs continuously across tiles; warp 1 issues
// tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM accumulators, so the
// epilogue of tile i overlaps the MMAs of tile i+1; warps 2-9 drain TMEM
// (tcgen05.ld; two warps per 32-lane quarter, each half of the tile's
// columns), apply alpha / bias / ReLU, convert, write 32-row x 128-byte chunks
// into swizzled shared memory and store them with TMA (bulk groups, one 4 KB
// buffer per warp).  Eight draining warps keep the epilogue shorter than the
// MMAs of a tile when K is short (an LM head's K = 512).  With split-K the raw f32 partial sums go to the
// workspace through the same TMA-store path.
// SPL: which operands arrive as bf16 hi + lo planes of f32 values (bit 0: A,
// bit 1: B); the others are bf16 as given.
template <int BN, int SPL = 0>
struct PcCfg {
  static constexpr int A_BYTES = 128 * 128;  // 128 rows x 64 bf16
  static constexpr int B_BYTES = BN * 128;
  static constexpr int AL_OFF = A_BYTES + B_BYTES;                          // [A | B | A lo | B lo]
  static constexpr int BL_OFF = AL_OFF + ((SPL & 1) ? A_BYTES : 0);
  static constexpr int STAGE = BL_OFF + ((SPL & 2) ? B_BYTES : 0);
  static constexpr int STAGES = (192 * 1024 / STAGE) > 8 ? 8 : (192 * 1024 / STAGE);
  static constexpr int EPI_BYTES = 8 * 4096;  // 8 epilogue warps x (32 rows x 128 B)
  static constexpr int SMEM = STAGES * STAGE + EPI_BYTES + 1024 + 256;
};

struct PersArgs {
  int M, N, K;
  int a_mn, b_mn;
  float alpha;
  const void* bias;
  int epi;  // 0 none, 1 bias, 2 bias+relu, 3 relu (ignored when out_ws)
  int tiles_m, tiles_n, batch, splits, kb_per_split, kb_all;
  int n_fast;  // 1: consecutive tiles step along N (fewer N tiles than M tiles)
  int group;   // > 1: grouped (swizzled) tile order, `group` M tiles per group
  int out_ws;  // 1: store raw f32 partials to the split-K workspace map
  int* err;
};

// alpha, bias and activation over one thread's CW consecutive outputs of a
// row, starting at column nc.  The mode tests sit outside the element loops:
// inside a fully unrolled loop they were two uniform branches per element,
// which made the plain case (alpha 1, no bias) cost several times its
// arithmetic.  Multiplying by an alpha of 1 is skipped (x * 1 == x exactly).
template <typename TO, int CW>
__device__ __forceinline__ void epilogue_row(float* v, const PersArgs& p, int nc) {
  if (p.alpha != 1.f) {
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] *= p.alpha;
  }
  if (p.epi == 1 || p.epi == 2) {
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] += nc + j < p.N ? load_bias<TO>(p.bias, nc + j) : 0.f;
  }
  if (p.epi >= 2) {
#pragma unroll
    for (int j = 0; j < CW; ++j) v[j] = fmaxf(v[j], 0.f);
  }
}


// f32 operands (SPL bits) arrive as bf16 hi and lo planes (split_planes); every
// K step issues hi*hi plus hi*lo for a split B and lo*hi for a split A (an
// operand that is bf16 already has no lo part: a mixed f32 x bf16 product
// takes two MMAs per step, two f32 operands three).
constexpr int kPersEpiWarps = 8;
constexpr int kPersThreads = 64 + 32 * kPersEpiWarps;
template <int BN, typename TO, int SPL>
__global__ void __launch_bounds__(kPersThreads, 1)
    gemm_tc_pers(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
                 const __grid_constant__ CUtensorMap tC, const __grid_constant__ CUtensorMap tAl,
                 const __grid_constant__ CUtensorMap tBl, PersArgs p) {
  pdl_wait();
  using Cfg = PcCfg<BN, SPL>;
  constexpr int S = Cfg::STAGES;
  constexpr int BK = 64;  // bf16 K elements per 128-byte row
  constexpr int E = 64;   // bf16 MN elements per 128-byte chunk
  constexpr int A_BYTES = Cfg::A_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* epi_smem = smem + S * Cfg::STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_smem + Cfg::EPI_BYTES);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2] accumulator ready
  uint64_t* tempty = tfull + 2;  // [2] accumulator drained
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);
  auto sA = [&](int s) { return smem + s * Cfg::STAGE; };
  auto sB = [&](int s) { return smem + s * Cfg::STAGE + A_BYTES; };
  auto sAl = [&](int s) { return smem + s * Cfg::STAGE + Cfg::AL_OFF; };
  auto sBl = [&](int s) { return smem + s * Cfg::STAGE + Cfg::BL_OFF; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_mn = p.tiles_m * p.tiles_n;
  const int num_tiles = tiles_mn * p.batch * p.splits;
  auto decode = [&](int t, int& m0, int& n0, int& bz, int& ks, int& kb0, int& nkb) {
    const int bs = t / tiles_mn, r = t - bs * tiles_mn;
    int mi, ni;
    if (p.group > 1) {
      // groups of `group` M tiles, N-major inside a group: the tiles resident at
      // once cover a squarish block of C, whose A and B panels stay in L2
      const int gsz = p.group * p.tiles_n;
      const int g = r / gsz, gm0 = g * p.group;
      const int gm = min(p.group, p.tiles_m - gm0);
      const int in = r - g * gsz;
      mi = gm0 + in % gm;
      ni = in / gm;
    } else if (p.n_fast) {
      ni = r % p.tiles_n;
      mi = r / p.tiles_n;
    } else {
      mi = r % p.tiles_m;
      ni = r / p.tiles_m;
    }
    m0 = mi * 128;
    n0 = ni * BN;
    bz = bs / p.splits;
    ks = bs - bz * p.splits;
    kb0 = ks * p.kb_per_split;
    nkb = max(0, min(p.kb_all, kb0 + p.kb_per_split) - kb0);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kPersEpiWarps);
    }
    *abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tA);
    tma_prefetch_desc(&tB);
    tma_prefetch_desc(&tC);
    if (SPL & 1) tma_prefetch_desc(&tAl);
    if (SPL & 2) tma_prefetch_desc(&tBl);
  }
  if (warp == 0) {
    tmem_alloc(tslot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
        int m0, n0, bz, ks, kb0, nkb;
        decode(t, m0, n0, bz, ks, kb0, nkb);
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % S, kb = kb0 + i;
          if (it >= S && !mbar_wait(&empty[s], ((it / S) + 1) & 1, abort, p.err, 111)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], Cfg::STAGE);
#pragma unroll
          for (int part = 0; part < (SPL ? 2 : 1); ++part) {
            const CUtensorMap* ma = part ? &tAl : &tA;
            const CUtensorMap* mb = part ? &tBl : &tB;
            uint8_t* da = part ? sAl(s) : sA(s);
            uint8_t* db = part ? sBl(s) : sB(s);
            if (part == 0 || (SPL & 1)) {
              if (!p.a_mn) {
                tma_load_3d(da, ma, &full[s], kb * BK, m0, bz);
              } else {
#pragma unroll
                for (int j = 0; j < 128 / E; ++j)
                  tma_load_3d(da + j * (BK * 128), ma, &full[s], m0 + j * E, kb * BK, bz);
              }
            }
            if (part == 0 || (SPL & 2)) {
              if (!p.b_mn) {
                tma_load_3d(db, mb, &full[s], kb * BK, n0, bz);
              } else {
#pragma unroll
                for (int j = 0; j < BN / E; ++j)
                  tma_load_3d(db + j * (BK * 128), mb, &full[s], n0 + j * E, kb * BK, bz);
              }
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = umma_idesc(1u, (uint32_t)p.a_mn, (uint32_t)p.b_mn, BN, 128);
      constexpr uint32_t KSTEP_MN = 16 * 128;  // bytes per K=16 step, MN-major
      auto adesc = [&](uint32_t base, int kk) {
        return p.a_mn ? umma_desc(base + kk * KSTEP_MN, BK * 128, 1024)
                      : umma_desc(base + kk * 32, 16, 1024);
      };
      auto bdesc = [&](uint32_t base, int kk) {
        return p.b_mn ? umma_desc(base + kk * KSTEP_MN, BK * 128, 1024)
                      : umma_desc(base + kk * 32, 16, 1024);
      };
      int it = 0, tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x, ++tl) {
        int m0, n0, bz, ks, kb0, nkb;
        decode(t, m0, n0, bz, ks, kb0, nkb);
        const int acc = tl & 1;
        if (tl >= 2 && !mbar_wait(&tempty[acc], ((tl >> 1) + 1) & 1, abort, p.err, 112)) break;
        tc_fence_after();
        const uint32_t dt = tmem + (uint32_t)(acc * BN);
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, abort, p.err, 113)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA(s)), b0 = smem_u32(sB(s));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_f16(dt, adesc(a0, kk), bdesc(b0, kk), idesc, (i | kk) != 0);
            if (SPL & 2) umma_f16(dt, adesc(a0, kk), bdesc(smem_u32(sBl(s)), kk), idesc, 1);
            if (SPL & 1) umma_f16(dt, adesc(smem_u32(sAl(s)), kk), bdesc(b0, kk), idesc, 1);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        if (nkb > 0) umma_commit(&tfull[acc]);
        else mbar_arrive(&tfull[acc]);
      }
    }
  } else {  // ---- warps 2..9: epilogue
    using TS = typename std::conditional<std::is_same<TO, float>::value, float, TO>::type;
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const int half = (warp - 2) >> 2;  // which half of the tile's column chunks
    uint8_t* stg = epi_smem + (warp - 2) * 4096;
    // this warp's column chunks [c_lo, c_hi) out of `n` (all of them for half 0
    // when there is a single chunk)
    auto chunks = [&](int n, int& c_lo, int& c_hi) {
      if (n < 2) { c_lo = 0; c_hi = half ? 0 : n; return; }
      c_lo = half * (n / 2);
      c_hi = half ? n : n / 2;
    };
    int tl = 0, nstore = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tl) {
      int m0, n0, bz, ks, kb0, nkb;
      decode(t, m0, n0, bz, ks, kb0, nkb);
      const int acc = tl & 1;
      bool ok = mbar_wait(&tfull[acc], (tl >> 1) & 1, abort, p.err, 114);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const int rowbase = m0 + q * 32;
      const int zc = p.out_ws ? bz * p.splits + ks : bz;
      if (p.out_ws) {
        // raw f32 partial sums: 32 columns per 128-byte chunk
        int c_lo, c_hi;
        chunks(BN / 32, c_lo, c_hi);
#pragma unroll 1
        for (int c = c_lo; c < c_hi; ++c) {
          const int nc = n0 + c * 32;
          if (nc >= p.N || rowbase >= p.M) continue;
          float v[32];
          if (nkb > 0) {
            tmem_ld32(trow + (uint32_t)(c * 32), v);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
          uint8_t* buf = stg;  // its previous store must have read it
          if (lane == 0 && nstore >= 1) bulk_wait_group_read<0>();
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(buf + lane * 128 + ((u ^ (lane & 7)) << 4)) =
                make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tC, buf, nc, rowbase, zc);
            bulk_commit_group();
          }
          ++nstore;
        }
      } else {
        constexpr int CW = 128 / (int)sizeof(TO);  // output columns per 128-byte chunk
        int c_lo, c_hi;
        chunks(BN / CW, c_lo, c_hi);
#pragma unroll 1
        for (int c = c_lo; c < c_hi; ++c) {
          const int nc = n0 + c * CW;
          if (nc >= p.N || rowbase >= p.M) continue;
          float v[CW];
          if (nkb > 0) {
            tmem_ld32(trow + (uint32_t)(c * CW), v);
            if (CW == 64) tmem_ld32(trow + (uint32_t)(c * CW + 32), v + 32);
          } else {
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] = 0.f;
          }
          epilogue_row<TO, CW>(v, p, nc);
          uint8_t* buf = stg;  // its previous store must have read it
          if (lane == 0 && nstore >= 1) bulk_wait_group_read<0>();
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            uint4 w;
            if (sizeof(TO) == 4) {
              w = make_uint4(__float_as_uint(v[4 * u]), __float_as_uint(v[4 * u + 1]),
                             __float_as_uint(v[4 * u + 2]), __float_as_uint(v[4 * u + 3]));
            } else {
              auto pk = [&](int j) {
                __nv_bfloat162 h = __floats2bfloat162_rn(v[j], v[j + 1]);
                return *reinterpret_cast<uint32_t*>(&h);
              };
              w = make_uint4(pk(8 * u), pk(8 * u + 2), pk(8 * u + 4), pk(8 * u + 6));
            }
            *reinterpret_cast<uint4*>(buf + lane * 128 + ((u ^ (lane & 7)) << 4)) = w;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tC, buf, nc, rowbase, zc);
            bulk_commit_group();
          }
          ++nstore;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (*abort && threadIdx.x == 0) {
    // let TMA copies already in flight land before the CTA's shared memory goes away
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 2000000ull) {
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

// Two-SM persistent bf16 GEMM: a cluster of two CTAs (a pair, on the two SMs
// of one TPC) computes 256 x 256 output tiles with tcgen05.mma.cta_group::2.
// Each CTA loads its own 128 rows of A and 128 of B's 256 columns per k-block
// (32 KB instead of the one-SM tile's 48 KB for 128 x 256 outputs), so a tile
// needs a third fewer operand bytes per SM, and the six-stage ring holds
// 192 KB in flight.  Roles as in gemm_tc_pers: warp 0 of each CTA streams its
// halves (both CTAs' loads complete on the rank-0 CTA's stage barrier, which
// rank 0 arms with the pair's byte count); warp 1 of rank 0 issues the MMAs
// (M = 256, N = 256, K = 16) into one of two TMEM accumulators and commits
// stage and accumulator barriers to both CTAs; warps 2-9 of each CTA drain
// their CTA's 128 accumulator rows and report on rank 0's barrier.  All
// waits are bounded.
struct PairCfg {
  static constexpr int A_BYTES = 128 * 128;  // this CTA's 128 rows x 64 bf16
  static constexpr int B_BYTES = 128 * 128;  // 128 of the tile's 256 columns x 64 bf16
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = 6;
  static constexpr int EPI_BYTES = 8 * 4096;  // 4 KB of output staging per epilogue warp
  static constexpr int SMEM = STAGES * STAGE + EPI_BYTES + 1024 + 256;
  static_assert(SMEM <= 232448, "shared memory above the 227 KB per-block limit");
};

template <typename TO>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPersThreads, 1)
    gemm_tc_pair(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
                 const __grid_constant__ CUtensorMap tC, PersArgs p) {
  pdl_wait();
  using Cfg = PairCfg;
  constexpr int S = Cfg::STAGES;
  constexpr int BN = 256;  // the pair tile's columns (each CTA loads half of B)
  constexpr int BK = 64;
  constexpr int E = 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* epi_smem = smem + S * Cfg::STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_smem + Cfg::EPI_BYTES);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2] accumulator ready (both CTAs)
  uint64_t* tempty = tfull + 2;  // [2] accumulator drained (rank 0: both CTAs' warps)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);
  auto sA = [&](int s) { return smem + s * Cfg::STAGE; };
  auto sB = [&](int s) { return smem + s * Cfg::STAGE + Cfg::A_BYTES; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)cluster_rank();
  const int pair = (int)blockIdx.x >> 1, npairs = (int)gridDim.x >> 1;
  const int tiles_mn = p.tiles_m * p.tiles_n;
  const int num_tiles = tiles_mn * p.batch * p.splits;  // work units: tiles x K splits
  auto decode = [&](int t, int& m0, int& n0, int& bz, int& ks, int& kb0, int& nkb) {
    const int bs = t / tiles_mn, r = t - bs * tiles_mn;
    int mi, ni;
    if (p.group > 1) {
      const int gsz = p.group * p.tiles_n;
      const int g = r / gsz, gm0 = g * p.group;
      const int gm = min(p.group, p.tiles_m - gm0);
      const int in = r - g * gsz;
      mi = gm0 + in % gm;
      ni = in / gm;
    } else if (p.n_fast) {
      ni = r % p.tiles_n;
      mi = r / p.tiles_n;
    } else {
      mi = r % p.tiles_m;
      ni = r / p.tiles_m;
    }
    m0 = mi * 256;
    n0 = ni * BN;
    bz = bs / p.splits;
    ks = bs - bz * p.splits;
    kb0 = ks * p.kb_per_split;
    nkb = max(0, min(p.kb_all, kb0 + p.kb_per_split) - kb0);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kPersEpiWarps);
    }
    *abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tA);
    tma_prefetch_desc(&tB);
    tma_prefetch_desc(&tC);
  }
  if (warp == 0) {
    tmem_alloc_pair(tslot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other's
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer (both CTAs)
      int it = 0;
      bool ok = true;
      for (int t = pair; ok && t < num_tiles; t += npairs) {
        int m0, n0, bz, ks, kb0, nkb;
        decode(t, m0, n0, bz, ks, kb0, nkb);
        const int mr = m0 + rank * 128, nr = n0 + rank * 128;  // this CTA's rows / columns
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % S, kb = kb0 + i;
          if (it >= S && !mbar_wait(&empty[s], ((it / S) + 1) & 1, abort, p.err, 121)) {
            ok = false;
            break;
          }
          const uint32_t bar = pair_leader_addr(smem_u32(&full[s]));
          if (rank == 0) mbar_expect_tx(&full[s], 2 * Cfg::STAGE);
          if (!p.a_mn) {
            tma_load_3d_pair(sA(s), &tA, bar, kb * BK, mr, bz);
          } else {
#pragma unroll
            for (int j = 0; j < 128 / E; ++j) tma_load_3d_pair(sA(s) + j * (BK * 128), &tA, bar, mr + j * E, kb * BK, bz);
          }
          if (!p.b_mn) {
            tma_load_3d_pair(sB(s), &tB, bar, kb * BK, nr, bz);
          } else {
#pragma unroll
            for (int j = 0; j < 128 / E; ++j) tma_load_3d_pair(sB(s) + j * (BK * 128), &tB, bar, nr + j * E, kb * BK, bz);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {  // ---- MMA issuer (the pair's rank 0)
      const uint32_t idesc = umma_idesc(1u, (uint32_t)p.a_mn, (uint32_t)p.b_mn, BN, 256);
      constexpr uint32_t KSTEP_MN = 16 * 128;
      auto desc = [&](uint32_t base, int kk, int mn) {
        return mn ? umma_desc(base + kk * KSTEP_MN, BK * 128, 1024) : umma_desc(base + kk * 32, 16, 1024);
      };
      int it = 0, tl = 0;
      bool ok = true;
      for (int t = pair; ok && t < num_tiles; t += npairs, ++tl) {
        int m0, n0, bz, ks, kb0, nkb;
        decode(t, m0, n0, bz, ks, kb0, nkb);
        const int acc = tl & 1;
        if (tl >= 2 && !mbar_wait(&tempty[acc], ((tl >> 1) + 1) & 1, abort, p.err, 122)) break;
        tc_fence_after();
        const uint32_t dt = tmem + (uint32_t)(acc * BN);
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, abort, p.err, 123)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA(s)), b0 = smem_u32(sB(s));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_pair(dt, desc(a0, kk, p.a_mn), desc(b0, kk, p.b_mn), idesc, (i | kk) != 0);
          umma_commit_pair(&empty[s]);
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc]);
      }
    }
  } else {  // ---- warps 2..9 of both CTAs: epilogue of this CTA's 128 rows
    // Each warp drains 32 rows x 128 columns per tile, one 128-byte-wide box
    // (4 KB of staging) at a time: the accumulator is released as soon as its
    // last columns are in registers, and the staging is rewritten once the
    // previous box's store has read it.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stg = epi_smem + (warp - 2) * 4096;
    constexpr int CW = 128 / (int)sizeof(TO);  // output columns per 128-byte box
    constexpr int NB = (BN / 2) / CW;          // boxes per warp and tile: 2 (bf16), 4 (f32)
    int tl = 0;
    bool pending = false;
    for (int t = pair; t < num_tiles; t += npairs, ++tl) {
      int m0, n0, bz, ks, kb0, nkb;
      decode(t, m0, n0, bz, ks, kb0, nkb);
      const int zc = bz * p.splits + ks;  // output slice: the batch entry, or its split's partials
      const int acc = tl & 1;
      bool ok = mbar_wait(&tfull[acc], (tl >> 1) & 1, abort, p.err, 124);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const int rowbase = m0 + rank * 128 + q * 32;
#pragma unroll 1
      for (int i = 0; i < NB; ++i) {
        const int c = half * NB + i;
        uint32_t raw[CW];
        tmem_ld32_async(trow + (uint32_t)(c * CW), raw);
        if (CW == 64) tmem_ld32_async(trow + (uint32_t)(c * CW + 32), raw + 32);
        tmem_wait_ld();
        if (nkb == 0) {  // an empty K range: the accumulator was never written
#pragma unroll
          for (int j = 0; j < CW; ++j) raw[j] = 0u;
        }
        if (i == NB - 1) {  // every column of the accumulator is read
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(pair_leader_addr(smem_u32(&tempty[acc])));
        }
        const int nc = n0 + c * CW;
        float v[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) v[j] = __uint_as_float(raw[j]);
        epilogue_row<TO, CW>(v, p, nc);
        if (pending) {  // the previous box's store must have read the staging
          if (lane == 0) bulk_wait_group_read<0>();
          __syncwarp();
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          uint4 w;
          if (sizeof(TO) == 4) {
            w = make_uint4(__float_as_uint(v[4 * u]), __float_as_uint(v[4 * u + 1]),
                           __float_as_uint(v[4 * u + 2]), __float_as_uint(v[4 * u + 3]));
          } else {
            auto pk = [&](int j) {
              __nv_bfloat162 h = __floats2bfloat162_rn(v[j], v[j + 1]);
              return *reinterpret_cast<uint32_t*>(&h);
            };
            w = make_uint4(pk(8 * u), pk(8 * u + 2), pk(8 * u + 4), pk(8 * u + 6));
          }
          *reinterpret_cast<uint4*>(stg + lane * 128 + ((u ^ (lane & 7)) << 4)) = w;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (nc < p.N && rowbase < p.M) tma_store_3d(&tC, stg, nc, rowbase, zc);
          bulk_commit_group();
        }
        pending = true;
      }
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (*abort && threadIdx.x == 0) {
    // let copies and MMAs already in flight land before shared memory / TMEM go away
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 2000000ull) {
    }
  }
  cluster_sync_all();  // neither CTA leaves while the other may still signal it
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 2 * BN);
  }
}

// SIMT fallback: 64x64 tile, 256 threads, 4x4 outputs per thread, f32 FMA.
template <typename TI, typename TO>
__global__ void __launch_bounds__(256)
    gemm_simt(const TI* __restrict__ A, const TI* __restrict__ B, TO* __restrict__ C,
              const void* bias, int M, int N, int K, int64_t sAb, int64_t sAm, int64_t sAk,
              int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, int64_t sCb, float alpha,
              int epi, int splits, int kchunk, float* __restrict__ ws) {
  pdl_wait();
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  const int bz = blockIdx.z / splits, ks = blockIdx.z % splits;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  A += (int64_t)bz * sAb;
  B += (int64_t)bz * sBb;
  const int kbeg = ks * kchunk, kend = min(K, kbeg + kchunk);
  float acc[4][4] = {};
  for (int k0 = kbeg; k0 < kend; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int mm = i / 16, kk = i % 16;  // A tile [64 m][16 k]
      const int gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < kend) ? Io<TI>::to_f(A[gm * sAm + gk * sAk]) : 0.f;
      const int kk2 = i / 64, nn = i % 64;  // B tile [16 k][64 n]
      const int gk2 = k0 + kk2, gn = n0 + nn;
      Bs[kk2][nn] = (gk2 < kend && gn < N) ? Io<TI>::to_f(B[gk2 * sBk + gn * sBn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      if (splits > 1) {
        ws[((int64_t)blockIdx.z * M + m) * N + n] = acc[i][j];
        continue;
      }
      float x = acc[i][j] * alpha;
      if (epi == 1 || epi == 2) x += Io<TO>::to_f(reinterpret_cast<const TO*>(bias)[n]);
      if (epi >= 2) x = fmaxf(x, 0.f);
      store_out<TO>(C + (int64_t)bz * sCb + (int64_t)m * ldc + n, x);
    }
  }
}

// Narrow outputs (N <= 16, e.g. the 10-class logits and their gradients): one
// thread per output row keeps all N accumulators; each block stages a 64-deep
// slab of A (read along its contiguous dimension, so both A and A^T load
// coalesced) and of B in shared memory.  K is split over blocks until the grid
// covers the GPU (partials summed in split order by splitk_reduce1).
template <typename TI, typename TO, int NMAX>
__global__ void __launch_bounds__(128)
    gemm_skinny(const TI* __restrict__ A, const TI* __restrict__ B, TO* __restrict__ C,
                const void* bias, int M, int N, int K, int64_t sAb, int64_t sAm, int64_t sAk,
                int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, int64_t sCb, float alpha,
                int epi, int splits, int kchunk, float* __restrict__ ws) {
  pdl_wait();
  __shared__ float As[64][129];  // [k][m]: conflict-free column reads and either-major fills
  __shared__ float Bs[64][NMAX];
  const int bz = blockIdx.z / splits, ks = blockIdx.z % splits;
  const int m0 = blockIdx.x * 128;
  const int m = m0 + threadIdx.x;
  A += (int64_t)bz * sAb;
  B += (int64_t)bz * sBb;
  const int kbeg = ks * kchunk, kend = min(K, kbeg + kchunk);
  float acc[NMAX];
#pragma unroll
  for (int n = 0; n < NMAX; ++n) acc[n] = 0.f;
  for (int k0 = kbeg; k0 < kend; k0 += 64) {
    // A tile (64 k x 128 m), read along whichever of k / m is contiguous
    if (sAk == 1) {
      for (int i = threadIdx.x; i < 64 * 128; i += 128) {
        const int mm = i >> 6, kk = i & 63, gm = m0 + mm, gk = k0 + kk;
        As[kk][mm] = (gm < M && gk < kend) ? Io<TI>::to_f(A[(int64_t)gm * sAm + gk]) : 0.f;
      }
    } else {
      for (int i = threadIdx.x; i < 64 * 128; i += 128) {
        const int kk = i >> 7, mm = i & 127, gm = m0 + mm, gk = k0 + kk;
        As[kk][mm] =
            (gm < M && gk < kend) ? Io<TI>::to_f(A[(int64_t)gm * sAm + (int64_t)gk * sAk]) : 0.f;
      }
    }
    for (int i = threadIdx.x; i < 64 * NMAX; i += 128) {
      const int kk = i / NMAX, n = i % NMAX, gk = k0 + kk;
      Bs[kk][n] = (gk < kend && n < N) ? Io<TI>::to_f(B[(int64_t)gk * sBk + (int64_t)n * sBn]) : 0.f;
    }
    __syncthreads();
    const int kn = min(64, kend - k0);
    for (int kk = 0; kk < kn; ++kk) {
      const float a = As[kk][threadIdx.x];
#pragma unroll
      for (int n = 0; n < NMAX; ++n) acc[n] = fmaf(a, Bs[kk][n], acc[n]);
    }
    __syncthreads();
  }
  auto finish = [&](float* v) {
    for (int n = 0; n < N && n < NMAX; ++n) {
      float x = v[n] * alpha;
      if (epi == 1 || epi == 2) x += Io<TO>::to_f(reinterpret_cast<const TO*>(bias)[n]);
      if (epi >= 2) x = fmaxf(x, 0.f);
      store_out<TO>(C + (int64_t)bz * sCb + (int64_t)m * ldc + n, x);
    }
  };
  if (m >= M) return;
  if (splits == 1) {
    finish(acc);
    return;
  }
  // split-K partials, summed in split order by splitk_reduce1
  for (int n = 0; n < N && n < NMAX; ++n) ws[((int64_t)blockIdx.z * M + m) * N + n] = acc[n];
}

// Split-K plan: when the output tiles alone cannot fill the GPU, the K loop is
// divided so that about two CTAs per SM run; each split keeps at least
// `min_blocks` k-blocks so the partial-sum traffic stays small next to the
// operand traffic.
struct SplitPlan {
  int splits = 1, per_split = 1;
};
SplitPlan plan_splits(int64_t tiles, int kblocks, int min_blocks, int64_t batch) {
  SplitPlan sp;
  sp.per_split = std::max(kblocks, 1);
  const int64_t target = 2 * (int64_t)num_sms();
  if (tiles >= num_sms() || kblocks < 2 * min_blocks) return sp;
  int64_t want = (target + tiles - 1) / tiles;
  want = std::min<int64_t>(want, kblocks / min_blocks);
  want = std::min<int64_t>(want, 64);
  want = std::min<int64_t>(want, 65535 / std::max<int64_t>(batch, 1));
  if (want <= 1) return sp;
  sp.per_split = (int)((kblocks + want - 1) / want);
  sp.splits = (kblocks + sp.per_split - 1) / sp.per_split;
  return sp;
}

// The order in which a persistent grid walks its output tiles.  When one
// operand's whole panel (all its rows of one batch entry) is small enough to
// stay in L2 (24 MB) while the other streams past, the walk runs along that
// operand's tiles fastest: it stays resident and each panel of the other is
// read from memory once (the LM head's 16 MB of activations against 32 MB of
// weights and 1 GB of logits written meanwhile).  Otherwise groups of `group`
// M tiles are walked N-major, so the tiles resident at once cover a squarish
// block of C whose A and B panels stay in L2.
void tile_order(int64_t M, int64_t N, int64_t K, int64_t tiles_m, int64_t tiles_n, int group,
                PersArgs& p) {
  const double a_bytes = 2.0 * M * K, b_bytes = 2.0 * N * K;
  constexpr double kResident = 24.0 * (1 << 20);
  if (std::min(a_bytes, b_bytes) <= kResident) {
    p.n_fast = b_bytes <= a_bytes ? 1 : 0;  // N fastest: B is the resident panel
    p.group = 1;
    return;
  }
  p.n_fast = tiles_n <= tiles_m ? 1 : 0;
  p.group = (tiles_m >= 2 * group && tiles_n >= 16) ? group : 1;
}

// Where split-K partial sums live.  b200_gemm takes stream-ordered memory from
// the CUDA memory pool (cudaMallocAsync / cudaFreeAsync on the launch stream);
// a caller may instead lend a fixed buffer.
// Returned by the launchers (before any launch) when a Scratch is only
// measuring how much workspace a call needs.
constexpr int kWorkspaceQueried = 1000;

struct Scratch {
  void* lent = nullptr;  // one fixed buffer for split-K partials (b200_gemm_noalloc)
  size_t lent_bytes = 0;
  bool has_arena = false;  // caller's workspace, carved in 256-byte units (b200_gemm_ws)
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0, arena_used = 0;
  bool query = false;   // record sizes only (b200_gemm_workspace_bytes)
  size_t queried = 0;
  int* err = nullptr;  // bounded-wait error word; nullptr: device_error_word()
  void* owned[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  int n_owned = 0;
  cudaStream_t owned_stream = nullptr;
  int get(size_t bytes, cudaStream_t st, float** out) {
    if (lent) {
      if (bytes > lent_bytes)
        return set_error(B200_ERR_INVALID, "gemm: split-K needs " + std::to_string(bytes) +
                                               " bytes of scratch, the fixed scratch array holds " +
                                               std::to_string(lent_bytes));
      *out = static_cast<float*>(lent);
      return B200_OK;
    }
    return get_owned(bytes, st, reinterpret_cast<void**>(out));
  }
  // Workspace for this call: carved from the caller's arena, or stream-ordered
  // memory from the CUDA pool released when the call returns (after its
  // kernels in stream order).
  int get_owned(size_t bytes, cudaStream_t st, void** out) {
    const size_t rounded = (bytes + 255) / 256 * 256;
    // Under b200_gemm_noalloc the only memory is the fixed array: a path that
    // would need any other buffer is refused, never served by an allocation.
    if (lent)
      return set_error(B200_ERR_UNSUPPORTED,
                       "gemm_noalloc: this operand layout needs a workspace buffer beyond the "
                       "fixed split-K array");
    if (query) {
      queried += rounded;
      *out = reinterpret_cast<void*>((uintptr_t)4096);  // encodes descriptors; never launched
      return B200_OK;
    }
    if (has_arena) {
      if (arena_used + rounded > arena_bytes)
        return set_error(B200_ERR_INVALID, "gemm: workspace of " + std::to_string(arena_bytes) +
                                               " bytes is too small");
      *out = arena + arena_used;
      arena_used += rounded;
      return B200_OK;
    }
    if (n_owned == 6) return set_error(B200_ERR_INVALID, "gemm: too many scratch buffers");
    B200_CUDA_TRY(cudaMallocAsync(&owned[n_owned], bytes, st));
    owned_stream = st;
    *out = owned[n_owned++];
    return B200_OK;
  }
  ~Scratch() {
    for (int i = 0; i < n_owned; ++i) cudaFreeAsync(owned[i], owned_stream);
  }
};

// f32 -> bf16 hi (rounded) and lo (rounded residual) planes, same element
// offsets: x ~= hi + lo to ~2^-16 relative.  blockIdx.y selects one of two
// operands (both GEMM operands in one launch).
struct PlaneJob {
  const float* x;
  __nv_bfloat16* hi;
  __nv_bfloat16* lo;
  int64_t n;
};
__global__ void __launch_bounds__(256) split_planes(PlaneJob j0, PlaneJob j1) {
  pdl_wait();
  const PlaneJob& j = blockIdx.y ? j1 : j0;
  const float* __restrict__ x = j.x;
  __nv_bfloat16* __restrict__ hi = j.hi;
  __nv_bfloat16* __restrict__ lo = j.lo;
  const int64_t n = j.n;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 4;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 4 <= n && ((reinterpret_cast<uintptr_t>(x + i) | reinterpret_cast<uintptr_t>(hi + i) |
                        reinterpret_cast<uintptr_t>(lo + i)) & 7) == 0 &&
        ((reinterpret_cast<uintptr_t>(x + i)) & 15) == 0) {
      const float4 v = *reinterpret_cast<const float4*>(x + i);
      const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
      const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
      const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - f0.x, v.y - f0.y);
      const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - f1.x, v.w - f1.y);
      uint2 hv, lv;
      hv.x = *reinterpret_cast<const uint32_t*>(&h0);
      hv.y = *reinterpret_cast<const uint32_t*>(&h1);
      lv.x = *reinterpret_cast<const uint32_t*>(&l0);
      lv.y = *reinterpret_cast<const uint32_t*>(&l1);
      *reinterpret_cast<uint2*>(hi + i) = hv;
      *reinterpret_cast<uint2*>(lo + i) = lv;
    } else {
      for (int64_t k = i; k < n && k < i + 4; ++k) {
        const __nv_bfloat16 h = __float2bfloat16_rn(x[k]);
        hi[k] = h;
        lo[k] = __float2bfloat16_rn(x[k] - __bfloat162float(h));
      }
    }
  }
}

// hi + lo bf16 planes -> f32 (the fallback when planes given by the caller
// cannot feed the persistent kernel).
__global__ void __launch_bounds__(256)
    join_planes(const __nv_bfloat16* __restrict__ hi, const __nv_bfloat16* __restrict__ lo,
                float* __restrict__ y, int64_t n) {
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __bfloat162float(hi[i]) + __bfloat162float(lo[i]);
}

// bf16 -> f32, element for element (the fallback for a mixed-type product).
__global__ void __launch_bounds__(256)
    widen_bf16(const __nv_bfloat16* __restrict__ x, float* __restrict__ y, int64_t n) {
  pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __bfloat162float(x[i]);
}

// Sums the split-K partials in a fixed order (deterministic) and applies the
// epilogue: C[b,m,n] = epi(alpha * sum_s ws[b*splits+s][m][n] (+ bias[n])).
// One thread per 4 consecutive outputs of a row (N % 4 == 0; rows = batch * M
// of N outputs each); partials read as float4.
template <typename TO>
__global__ void __launch_bounds__(256)
    splitk_reduce(const float* __restrict__ ws, TO* __restrict__ C, const void* bias, int batch,
                  int M, int N, int splits, int64_t ldc, int64_t sCb, float alpha, int epi) {
  pdl_wait();
  const int nq = N >> 2;
  const int64_t total = (int64_t)batch * M * nq;
  const int64_t mn_all = (int64_t)M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / nq;  // b * M + m
    const int n = (int)(i - row * nq) * 4;
    const int64_t b = row / M;
    const int m = (int)(row - b * M);
    const float* src = ws + b * splits * mn_all + (int64_t)m * N + n;
    float4 x = *reinterpret_cast<const float4*>(src);
    // unrolled: the loads of 8 splits are in flight together, the sums stay
    // in split order
#pragma unroll 8
    for (int k = 1; k < splits; ++k) {
      const float4 y = *reinterpret_cast<const float4*>(src + (int64_t)k * mn_all);
      x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
    }
    float v[4] = {x.x * alpha, x.y * alpha, x.z * alpha, x.w * alpha};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (epi == 1 || epi == 2) v[j] += Io<TO>::to_f(reinterpret_cast<const TO*>(bias)[n + j]);
      if (epi >= 2) v[j] = fmaxf(v[j], 0.f);
    }
    TO* dst = C + b * sCb + (int64_t)m * ldc + n;
#pragma unroll
    for (int j = 0; j < 4; ++j) store_out<TO>(dst + j, v[j]);
  }
}
// Any N: one thread per output.
template <typename TO>
__global__ void __launch_bounds__(256)
    splitk_reduce1(const float* __restrict__ ws, TO* __restrict__ C, const void* bias, int batch,
                   int M, int N, int splits, int64_t ldc, int64_t sCb, float alpha, int epi) {
  pdl_wait();
  const int64_t total = (int64_t)batch * M * N;
  const int64_t mn_all = (int64_t)M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / mn_all, mn = i - b * mn_all;
    const int m = (int)(mn / N), n = (int)(mn - (int64_t)m * N);
    const float* src = ws + b * splits * mn_all + mn;
    float x = 0.f;
#pragma unroll 8
    for (int k = 0; k < splits; ++k) x += src[(int64_t)k * mn_all];
    x *= alpha;
    if (epi == 1 || epi == 2) x += Io<TO>::to_f(reinterpret_cast<const TO*>(bias)[n]);
    if (epi >= 2) x = fmaxf(x, 0.f);
    store_out<TO>(C + b * sCb + (int64_t)m * ldc + n, x);
  }
}
template <typename TO>
int launch_splitk_reduce(const float* ws, TO* C, const void* bias, int64_t batch, int64_t M,
                         int64_t N, int splits, int64_t ldc, float alpha, int epi, cudaStream_t st) {
  if (N % 4 == 0) {
    const int64_t total = batch * M * (N / 4);
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
    B200_LAUNCH(splitk_reduce<TO>, dim3(blocks), dim3(256), 0, st, ws, C, bias, (int)batch, (int)M,
                (int)N, splits, ldc, M * ldc, alpha, epi);
  } else {
    const int64_t total = batch * M * N;
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
    B200_LAUNCH(splitk_reduce1<TO>, dim3(blocks), dim3(256), 0, st, ws, C, bias, (int)batch,
                (int)M, (int)N, splits, ldc, M * ldc, alpha, epi);
  }
  return B200_OK;
}

template <int BN, int ES, typename TO, bool SPLIT>
int launch_tc(const void* a, const void* b, void* c, const void* bias, int64_t batch, int64_t M,
              int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
              int64_t sBk, int64_t sBn, int64_t ldc, float alpha, int epi, int a_mn, int b_mn,
              cudaStream_t st, Scratch& scratch) {
  constexpr int BK = 128 / ES;
  constexpr int E = 128 / ES;
  CUtensorMap ta, tb;
  int rc;
  const bool atom32 = ES == 4;  // tf32 MN-major tiles need the 32-byte-unit swizzle
  // with a single batch the batch stride is never used: give TMA a legal one
  auto bstride = [&](int64_t s, int64_t outer_stride, int64_t outer_dim) -> uint64_t {
    const int64_t v = batch == 1 ? outer_stride * outer_dim : s;
    return (uint64_t)(((v * ES) + 15) / 16 * 16);
  };
  if (!a_mn) {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sAm * ES), bstride(sAb, sAm, M)};
    uint32_t box[3] = {(uint32_t)BK, 128, 1};
    rc = make_tmap(&ta, a, 3, dims, str, box, ES);
  } else {
    uint64_t dims[3] = {(uint64_t)M, (uint64_t)K, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sAk * ES), bstride(sAb, sAk, K)};
    uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
    rc = make_tmap(&ta, a, 3, dims, str, box, ES, atom32);
  }
  if (rc) return rc;
  if (!b_mn) {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sBn * ES), bstride(sBb, sBn, N)};
    uint32_t box[3] = {(uint32_t)BK, (uint32_t)BN, 1};
    rc = make_tmap(&tb, b, 3, dims, str, box, ES);
  } else {
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sBk * ES), bstride(sBb, sBk, K)};
    uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
    rc = make_tmap(&tb, b, 3, dims, str, box, ES, atom32);
  }
  if (rc) return rc;
  GemmArgs p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.alpha = alpha;
  p.bias = bias;
  p.epi = epi;
  p.c = c;
  p.ldc = ldc;
  p.sCb = M * ldc;
  p.err = scratch.err ? scratch.err : device_error_word();
  if (!p.err) return set_error(B200_ERR_CUDA, "could not allocate the device error word");
  const int smem = TcCfg<BN, ES, SPLIT>::SMEM;
  if (int rc2 = allow_dynamic_smem((const void*)gemm_tc<BN, ES, TO, SPLIT>, smem, "gemm_tc")) return rc2;
  const int64_t gx = (N + BN - 1) / BN, gy = (M + 127) / 128;
  const int KB_all = (int)((K + BK - 1) / BK);
  const SplitPlan sp = plan_splits(gx * gy * batch, KB_all, 4, batch);
  p.splits = sp.splits;
  p.kb_per_split = sp.per_split;
  p.ws = nullptr;
  if (sp.splits > 1) {
    if (int rc2 = scratch.get(sizeof(float) * (size_t)sp.splits * batch * M * N, st, &p.ws)) return rc2;
  }
  if (scratch.query) return kWorkspaceQueried;
  dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(batch * sp.splits));
  B200_LAUNCH(gemm_tc<BN, ES, TO, SPLIT>, grid, dim3(192), smem, st, ta, tb, p);
  if (sp.splits > 1)
    return launch_splitk_reduce<TO>(p.ws, (TO*)c, bias, batch, M, N, sp.splits, ldc, alpha, epi, st);
  return B200_OK;
}

// Persistent bf16 launch.  Returns B200_ERR_UNSUPPORTED (without launching)
// when the output cannot be stored with TMA (unaligned base or row pitch), so
// the caller can fall back to gemm_tc.
// Elements spanned by a strided operand (the highest offset + 1).
int64_t operand_span(int64_t batch, int64_t sb, int64_t r, int64_t sr, int64_t c, int64_t sc) {
  return (batch - 1) * sb + (r - 1) * sr + (c - 1) * sc + 1;
}

template <int BN, typename TO, int SPL = 0>
int launch_pers(const void* a, const void* b, void* c, const void* bias, int64_t batch, int64_t M,
                int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
                int64_t sBk, int64_t sBn, int64_t ldc, float alpha, int epi, int a_mn, int b_mn,
                cudaStream_t st, Scratch& scratch, const void* a_lo_in = nullptr,
                const void* b_lo_in = nullptr) {
  // a_lo_in / b_lo_in: the operand arrives split already (a / b are then its
  // bf16 hi plane)
  constexpr int ES = 2, BK = 64, E = 64;
  const int tiles_m = (int)((M + 127) / 128), tiles_n = (int)((N + BN - 1) / BN);
  const int KB_all = (int)((K + BK - 1) / BK);
  const SplitPlan sp = plan_splits((int64_t)tiles_m * tiles_n * batch, KB_all, 4, batch);
  const bool ws = sp.splits > 1;
  const int so = ws ? 4 : (int)sizeof(TO);
  if (ws ? (N * 4) % 16 != 0
         : (((uintptr_t)c & 15) != 0 || (ldc * so) % 16 != 0 || (batch > 1 && ((M * ldc * so) % 16) != 0)))
    return B200_ERR_UNSUPPORTED;
  auto bstride = [&](int64_t s, int64_t outer_stride, int64_t outer_dim) -> uint64_t {
    const int64_t v = batch == 1 ? outer_stride * outer_dim : s;
    return (uint64_t)(((v * ES) + 15) / 16 * 16);
  };
  // f32 operands: split into bf16 hi / lo planes with the same element strides
  // (a bf16 operand is read as it is and must meet the same 16-byte rules)
  const void* a_lo = nullptr;
  const void* b_lo = nullptr;
  int64_t na = 0, nb = 0;
  void *ah = nullptr, *al = nullptr, *bh = nullptr, *bl = nullptr;
  if (SPL) {
    if (scratch.lent) return B200_ERR_UNSUPPORTED;  // planes need memory: use the tf32 kernel
    if ((!(SPL & 1) || a_lo_in) && ((uintptr_t)a & 15)) return B200_ERR_UNSUPPORTED;
    if ((!(SPL & 2) || b_lo_in) && ((uintptr_t)b & 15)) return B200_ERR_UNSUPPORTED;
    if (((uintptr_t)a_lo_in & 15) || ((uintptr_t)b_lo_in & 15)) return B200_ERR_UNSUPPORTED;
    // the planes' row pitch (2-byte elements) must still be a multiple of 16 bytes
    auto ok16 = [](int64_t s) { return s == 1 || (s * 2) % 16 == 0; };
    if (!ok16(sAm) || !ok16(sAk) || !ok16(sBk) || !ok16(sBn) ||
        (batch > 1 && (!ok16(sAb) || !ok16(sBb))))
      return B200_ERR_UNSUPPORTED;
  }
  // all workspace first, so that a size query stops before anything launches
  float* wsp = nullptr;
  if (ws) {
    if (int rc2 = scratch.get(sizeof(float) * (size_t)sp.splits * batch * M * N, st, &wsp)) return rc2;
  }
  const bool split_a = (SPL & 1) && !a_lo_in, split_b = (SPL & 2) && !b_lo_in;
  if (split_a) {
    na = operand_span(batch, sAb, M, sAm, K, sAk);
    if (int r = scratch.get_owned(2 * (size_t)na, st, &ah)) return r;
    if (int r = scratch.get_owned(2 * (size_t)na, st, &al)) return r;
  }
  if (split_b) {
    nb = operand_span(batch, sBb, K, sBk, N, sBn);
    if (int r = scratch.get_owned(2 * (size_t)nb, st, &bh)) return r;
    if (int r = scratch.get_owned(2 * (size_t)nb, st, &bl)) return r;
  }
  if (scratch.query) return kWorkspaceQueried;
  if (split_a || split_b) {
    const unsigned g = (unsigned)std::min<int64_t>((std::max(na, nb) + 1023) / 1024, 148 * 4);
    const PlaneJob ja{(const float*)a, (__nv_bfloat16*)ah, (__nv_bfloat16*)al, (int64_t)na};
    const PlaneJob jb{(const float*)b, (__nv_bfloat16*)bh, (__nv_bfloat16*)bl, (int64_t)nb};
    if (split_a && split_b) B200_LAUNCH(split_planes, dim3(g, 2), dim3(256), 0, st, ja, jb);
    else B200_LAUNCH(split_planes, dim3(g, 1), dim3(256), 0, st, split_a ? ja : jb, ja);
  }
  if (SPL & 1) {
    a = split_a ? ah : a;
    a_lo = split_a ? al : a_lo_in;
  }
  if (SPL & 2) {
    b = split_b ? bh : b;
    b_lo = split_b ? bl : b_lo_in;
  }
  CUtensorMap ta, tb, tc, tal, tbl;
  int rc;
  if (!a_mn) {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sAm * ES), bstride(sAb, sAm, M)};
    uint32_t box[3] = {(uint32_t)BK, 128, 1};
    rc = make_tmap(&ta, a, 3, dims, str, box, ES);
  } else {
    uint64_t dims[3] = {(uint64_t)M, (uint64_t)K, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sAk * ES), bstride(sAb, sAk, K)};
    uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
    rc = make_tmap(&ta, a, 3, dims, str, box, ES);
  }
  if (rc) return rc;
  if (!b_mn) {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sBn * ES), bstride(sBb, sBn, N)};
    uint32_t box[3] = {(uint32_t)BK, (uint32_t)BN, 1};
    rc = make_tmap(&tb, b, 3, dims, str, box, ES);
  } else {
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sBk * ES), bstride(sBb, sBk, K)};
    uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
    rc = make_tmap(&tb, b, 3, dims, str, box, ES);
  }
  if (rc) return rc;
  tal = ta;  // (unused when the operand has no lo plane)
  tbl = tb;
  if (SPL & 1) {  // lo planes: same shapes and strides as the hi planes
    if (!a_mn) {
      uint64_t dims[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)batch};
      uint64_t str[2] = {(uint64_t)(sAm * ES), bstride(sAb, sAm, M)};
      uint32_t box[3] = {(uint32_t)BK, 128, 1};
      rc = make_tmap(&tal, a_lo, 3, dims, str, box, ES);
    } else {
      uint64_t dims[3] = {(uint64_t)M, (uint64_t)K, (uint64_t)batch};
      uint64_t str[2] = {(uint64_t)(sAk * ES), bstride(sAb, sAk, K)};
      uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
      rc = make_tmap(&tal, a_lo, 3, dims, str, box, ES);
    }
    if (rc) return rc;
  }
  if (SPL & 2) {
    if (!b_mn) {
      uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)batch};
      uint64_t str[2] = {(uint64_t)(sBn * ES), bstride(sBb, sBn, N)};
      uint32_t box[3] = {(uint32_t)BK, (uint32_t)BN, 1};
      rc = make_tmap(&tbl, b_lo, 3, dims, str, box, ES);
    } else {
      uint64_t dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)batch};
      uint64_t str[2] = {(uint64_t)(sBk * ES), bstride(sBb, sBk, K)};
      uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
      rc = make_tmap(&tbl, b_lo, 3, dims, str, box, ES);
    }
    if (rc) return rc;
  }
  PersArgs p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.alpha = alpha;
  p.bias = bias;
  p.epi = epi;
  p.tiles_m = tiles_m;
  p.tiles_n = tiles_n;
  p.batch = (int)batch;
  p.splits = sp.splits;
  p.kb_per_split = sp.per_split;
  p.kb_all = KB_all;
  tile_order(M, N, K, tiles_m, tiles_n, 16, p);
  p.out_ws = ws ? 1 : 0;
  p.err = scratch.err ? scratch.err : device_error_word();
  if (!p.err) return set_error(B200_ERR_CUDA, "could not allocate the device error word");
  if (ws) {
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)(batch * sp.splits)};
    uint64_t str[2] = {(uint64_t)(N * 4), (uint64_t)(M * N * 4)};
    uint32_t box[3] = {32, 32, 1};
    rc = make_tmap(&tc, wsp, 3, dims, str, box, 4);
  } else {
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)batch};
    const int64_t sc = batch == 1 ? M * ldc : M * ldc;
    uint64_t str[2] = {(uint64_t)(ldc * so), (uint64_t)(((sc * so) + 15) / 16 * 16)};
    uint32_t box[3] = {(uint32_t)(128 / so), 32, 1};
    rc = make_tmap(&tc, c, 3, dims, str, box, so);
  }
  if (rc) return rc;
  const int smem = PcCfg<BN, SPL>::SMEM;
  if (int rc2 = allow_dynamic_smem((const void*)gemm_tc_pers<BN, TO, SPL>, smem, "gemm_tc_pers")) return rc2;
  const int64_t num_tiles = (int64_t)tiles_m * tiles_n * batch * sp.splits;
  const unsigned grid = (unsigned)std::min<int64_t>(num_tiles, num_sms());
  B200_LAUNCH(gemm_tc_pers<BN, TO, SPL>, dim3(grid), dim3(kPersThreads), smem, st, ta, tb, tc, tal, tbl, p);
  if (ws)
    return launch_splitk_reduce<TO>(wsp, (TO*)c, bias, batch, M, N, sp.splits, ldc, alpha, epi, st);
  return B200_OK;
}

// The two-SM GEMM for bf16 operands: 256 x 256 tiles.  With fewer tiles than
// SM pairs, K is split so that about one (tile, K range) unit lands on each
// pair; the units write raw f32 partial sums which splitk_reduce adds in split
// order (alpha, bias and activation applied there).  Shapes that neither fill
// the pairs nor split stay on the one-SM kernel.  B200_GEMM_PAIR=0 turns it off.
bool use_pair() {
  static bool on = [] {
    const char* v = std::getenv("B200_GEMM_PAIR");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

// K splits for `tiles` pair tiles over `pairs` resident pairs: one unit per
// pair, or two when one leaves more than a tenth of the pairs idle; at least
// four k-blocks per unit.
SplitPlan plan_pair_splits(int64_t tiles, int kblocks, int64_t batch, int64_t pairs) {
  SplitPlan sp;
  sp.per_split = std::max(kblocks, 1);
  if (tiles >= pairs) return sp;
  auto plan = [&](int64_t want) {
    SplitPlan r;
    want = std::min<int64_t>({want, kblocks / 4, 64, 65535 / std::max<int64_t>(batch, 1)});
    if (want <= 1) return r;
    r.per_split = (int)((kblocks + want - 1) / want);
    r.splits = (kblocks + r.per_split - 1) / r.per_split;
    return r;
  };
  auto busy = [&](const SplitPlan& r) {  // fraction of pair slots doing work
    const int64_t units = tiles * r.splits;
    return (double)units / (double)(((units + pairs - 1) / pairs) * pairs);
  };
  const SplitPlan one = plan(pairs / tiles);
  if (one.splits > 1 && busy(one) >= 0.9) return one;
  const SplitPlan two = plan(2 * pairs / tiles);
  return busy(two) > busy(one) ? two : one;
}

template <typename TO>
int launch_pair(const void* a, const void* b, void* c, const void* bias, int64_t batch, int64_t M,
                int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb, int64_t sBk,
                int64_t sBn, int64_t ldc, float alpha, int epi, int a_mn, int b_mn, cudaStream_t st,
                Scratch& scratch) {
  constexpr int ES = 2, BK = 64, E = 64;
  const int smem = PairCfg::SMEM;
  // Clusters live inside one GPC, so fewer than num_sms / 2 pairs may fit at
  // once; a persistent grid larger than that would run a second wave.
  static const int max_pairs = [&] {
    if (allow_dynamic_smem((const void*)gemm_tc_pair<float>, smem, "gemm_tc_pair")) return num_sms() / 2;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(num_sms() & ~1);
    cfg.blockDim = dim3(kPersThreads);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)gemm_tc_pair<float>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    return n;
  }();
  const int64_t tiles_m = (M + 255) / 256, tiles_n = (N + 255) / 256;
  const int64_t tiles = tiles_m * tiles_n * batch;
  const int KB_all = (int)((K + BK - 1) / BK);
  if (M < 256 || N < 256 || tiles >= (1ll << 30)) return B200_ERR_UNSUPPORTED;
  const SplitPlan sp = plan_pair_splits(tiles, KB_all, batch, max_pairs);
  const bool ws = sp.splits > 1;
  if (!ws && tiles < max_pairs) return B200_ERR_UNSUPPORTED;
  const int so = (int)sizeof(TO);
  if (ws ? (N * 4) % 16 != 0
         : (((uintptr_t)c & 15) != 0 || (ldc * so) % 16 != 0 || (batch > 1 && ((M * ldc * so) % 16) != 0)))
    return B200_ERR_UNSUPPORTED;
  const size_t ws_bytes = ws ? sizeof(float) * (size_t)sp.splits * batch * M * N : 0;
  if (ws && scratch.lent && ws_bytes > scratch.lent_bytes) return B200_ERR_UNSUPPORTED;
  float* wsp = nullptr;
  if (ws) {
    if (int rc2 = scratch.get(ws_bytes, st, &wsp)) return rc2;
  }
  if (scratch.query) return kWorkspaceQueried;
  auto bstride = [&](int64_t s, int64_t outer_stride, int64_t outer_dim) -> uint64_t {
    const int64_t v = batch == 1 ? outer_stride * outer_dim : s;
    return (uint64_t)(((v * ES) + 15) / 16 * 16);
  };
  CUtensorMap ta, tb, tc;
  int rc;
  if (!a_mn) {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sAm * ES), bstride(sAb, sAm, M)};
    uint32_t box[3] = {(uint32_t)BK, 128, 1};
    rc = make_tmap(&ta, a, 3, dims, str, box, ES);
  } else {
    uint64_t dims[3] = {(uint64_t)M, (uint64_t)K, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sAk * ES), bstride(sAb, sAk, K)};
    uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
    rc = make_tmap(&ta, a, 3, dims, str, box, ES);
  }
  if (rc) return rc;
  if (!b_mn) {  // each CTA loads 128 of the tile's 256 columns
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sBn * ES), bstride(sBb, sBn, N)};
    uint32_t box[3] = {(uint32_t)BK, 128, 1};
    rc = make_tmap(&tb, b, 3, dims, str, box, ES);
  } else {
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sBk * ES), bstride(sBb, sBk, K)};
    uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
    rc = make_tmap(&tb, b, 3, dims, str, box, ES);
  }
  if (rc) return rc;
  if (ws) {  // partials: [batch * splits][M][N] f32
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)(batch * sp.splits)};
    uint64_t str[2] = {(uint64_t)(N * 4), (uint64_t)(M * N * 4)};
    uint32_t box[3] = {32, 32, 1};
    rc = make_tmap(&tc, wsp, 3, dims, str, box, 4);
  } else {
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(ldc * so), (uint64_t)(((M * ldc * so) + 15) / 16 * 16)};
    uint32_t box[3] = {(uint32_t)(128 / so), 32, 1};
    rc = make_tmap(&tc, c, 3, dims, str, box, so);
  }
  if (rc) return rc;
  PersArgs p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.alpha = ws ? 1.f : alpha;
  p.bias = ws ? nullptr : bias;
  p.epi = ws ? 0 : epi;
  p.tiles_m = (int)tiles_m;
  p.tiles_n = (int)tiles_n;
  p.batch = (int)batch;
  p.splits = sp.splits;
  p.kb_all = KB_all;
  p.kb_per_split = sp.per_split;
  tile_order(M, N, K, tiles_m, tiles_n, 8, p);
  p.out_ws = ws ? 1 : 0;
  p.err = scratch.err ? scratch.err : device_error_word();
  if (!p.err) return set_error(B200_ERR_CUDA, "could not allocate the device error word");
  const unsigned grid = (unsigned)(2 * std::min<int64_t>(tiles * sp.splits, max_pairs));
  if (ws) {
    if (int rc2 = allow_dynamic_smem((const void*)gemm_tc_pair<float>, smem, "gemm_tc_pair")) return rc2;
    B200_LAUNCH(gemm_tc_pair<float>, dim3(grid), dim3(kPersThreads), smem, st, ta, tb, tc, p);
    return launch_splitk_reduce<TO>(wsp, (TO*)c, bias, batch, M, N, sp.splits, ldc, alpha, epi, st);
  }
  if (int rc2 = allow_dynamic_smem((const void*)gemm_tc_pair<TO>, smem, "gemm_tc_pair")) return rc2;
  B200_LAUNCH(gemm_tc_pair<TO>, dim3(grid), dim3(kPersThreads), smem, st, ta, tb, tc, p);
  return B200_OK;
}

bool use_persistent() {
  static bool on = [] {
    const char* v = std::getenv("B200_GEMM_PERSISTENT");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

template <typename TI, typename TO>
int launch_simt(const void* a, const void* b, void* c, const void* bias, int64_t batch, int64_t M,
                int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
                int64_t sBk, int64_t sBn, int64_t ldc, float alpha, int epi, cudaStream_t st,
                Scratch& scratch) {
  if (N <= 16) {
    const int64_t gx = (M + 127) / 128;
    const SplitPlan sp = plan_splits(gx * batch, (int)((K + 63) / 64), 1, batch);
    float* ws = nullptr;
    if (sp.splits > 1) {
      if (int rc = scratch.get(sizeof(float) * (size_t)sp.splits * batch * M * N, st, &ws)) return rc;
    }
    if (scratch.query) return kWorkspaceQueried;
    dim3 grid((unsigned)gx, 1, (unsigned)(batch * sp.splits));
    B200_LAUNCH(gemm_skinny<TI, TO, 16>, grid, dim3(128), 0, st, (const TI*)a, (const TI*)b, (TO*)c,
                bias, (int)M, (int)N, (int)K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, M * ldc, alpha, epi,
                sp.splits, sp.per_split * 64, ws);
    if (sp.splits > 1)
      return launch_splitk_reduce<TO>(ws, (TO*)c, bias, batch, M, N, sp.splits, ldc, alpha, epi, st);
    return B200_OK;
  }
  const int64_t gx = (N + 63) / 64, gy = (M + 63) / 64;
  const SplitPlan sp = plan_splits(gx * gy * batch, (int)((K + 15) / 16), 8, batch);
  float* ws = nullptr;
  if (sp.splits > 1) {
    if (int rc = scratch.get(sizeof(float) * (size_t)sp.splits * batch * M * N, st, &ws)) return rc;
  }
  if (scratch.query) return kWorkspaceQueried;
  dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(batch * sp.splits));
  B200_LAUNCH(gemm_simt<TI, TO>, grid, dim3(256), 0, st, (const TI*)a, (const TI*)b, (TO*)c, bias,
              (int)M, (int)N, (int)K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, M * ldc, alpha, epi,
              sp.splits, sp.per_split * 16, ws);
  if (sp.splits > 1)
    return launch_splitk_reduce<TO>(ws, (TO*)c, bias, batch, M, N, sp.splits, ldc, alpha, epi, st);
  return B200_OK;
}

// f32 matmuls: 3xTF32 (default; f32-level accuracy) or 1xTF32 with
// B200_F32_MATMUL=tf32 (one MMA per step, ~1e-3 relative error).
bool f32_matmul_3x() {
  static bool x3 = [] {
    const char* v = std::getenv("B200_F32_MATMUL");
    return !(v && std::strcmp(v, "tf32") == 0);
  }();
  return x3;
}

bool force_simt() {
  static bool f = [] {
    const char* v = std::getenv("B200_GEMM_SIMT");
    return v && *v && std::strcmp(v, "0") != 0;
  }();
  return f;
}

}  // namespace
}  // namespace b200

namespace b200 {
namespace {
int gemm_dispatch(const void* a, const void* b, void* c, const void* bias, int64_t batch,
                  int64_t M, int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk,
                  int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, float alpha,
                  int in_dtype, int out_dtype, int epilogue, void* stream, Scratch& scratch) {
  B200_CHECK_ARG(a && b && c, "gemm: null operand");
  B200_CHECK_ARG(batch >= 1 && M >= 0 && N >= 0 && K >= 0, "gemm: bad shape");
  B200_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31) && batch < 65536,
                 "gemm: dimension too large");
  B200_CHECK_ARG(epilogue >= 0 && epilogue <= 3, "gemm: bad epilogue");
  B200_CHECK_ARG(!(epilogue == 1 || epilogue == 2) || bias, "gemm: epilogue needs a bias");
  B200_CHECK_ARG(in_dtype == B200_DT_F32 || in_dtype == B200_DT_BF16 ||
                     in_dtype == B200_GEMM_DT_A_F32_B_BF16 || in_dtype == B200_GEMM_DT_A_BF16_B_F32,
                 "gemm: in_dtype must be F32, BF16 or a mixed F32 x BF16 code");
  B200_CHECK_ARG(out_dtype == B200_DT_F32 || out_dtype == B200_DT_BF16, "gemm: out_dtype must be F32 or BF16");
  if (ldc <= 0) ldc = N;
  if (M == 0 || N == 0) return B200_OK;
  auto st = (cudaStream_t)stream;
  if (K == 0) {
    // An empty sum: C = 0 (relu(0) = 0).  C is batch*M rows of N elements,
    // ldc apart (the batch stride is M*ldc).  With a bias the result would be
    // the bias broadcast, which no caller asks for with K == 0.
    if (epilogue == 1 || epilogue == 2)
      return set_error(B200_ERR_UNSUPPORTED, "gemm: K == 0 with a bias epilogue is not supported");
    if (scratch.query) return B200_OK;
    const size_t es = out_dtype == B200_DT_BF16 ? 2 : 4;
    B200_CUDA_TRY(cudaMemset2DAsync(c, (size_t)ldc * es, 0, (size_t)N * es, (size_t)(batch * M), st));
    return B200_OK;
  }
  if (in_dtype == B200_GEMM_DT_A_F32_B_BF16 || in_dtype == B200_GEMM_DT_A_BF16_B_F32) {
    const bool a32 = in_dtype == B200_GEMM_DT_A_F32_B_BF16;
    const bool obf = out_dtype == B200_DT_BF16;
    // persistent kernel: the f32 operand as bf16 hi + lo planes, the bf16 one as given
    auto m16 = [](int64_t s) { return ((s * 2) & 15) == 0; };
    int a_mn = -1, b_mn = -1;
    if (sAk == 1 && m16(sAm) && (batch == 1 || m16(sAb))) a_mn = 0;
    else if (sAm == 1 && m16(sAk) && (batch == 1 || m16(sAb))) a_mn = 1;
    if (sBk == 1 && m16(sBn) && (batch == 1 || m16(sBb))) b_mn = 0;
    else if (sBn == 1 && m16(sBk) && (batch == 1 || m16(sBb))) b_mn = 1;
    if (!force_simt() && use_persistent() && f32_matmul_3x() && a_mn >= 0 && b_mn >= 0 && K * 2 >= 16) {
      int prc;
#define B200_PERSM(BN_, TO_)                                                                       \
  prc = a32 ? launch_pers<BN_, TO_, 1>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, \
                                       ldc, alpha, epilogue, a_mn, b_mn, st, scratch)              \
            : launch_pers<BN_, TO_, 2>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, \
                                       ldc, alpha, epilogue, a_mn, b_mn, st, scratch)
      if (N <= 64) { if (obf) B200_PERSM(64, __nv_bfloat16); else B200_PERSM(64, float); }
      else if (N <= 128) { if (obf) B200_PERSM(128, __nv_bfloat16); else B200_PERSM(128, float); }
      else { if (obf) B200_PERSM(256, __nv_bfloat16); else B200_PERSM(256, float); }
#undef B200_PERSM
      if (prc != B200_ERR_UNSUPPORTED) return prc;
    }
    // anything else: the bf16 operand widened to f32 (same element offsets), then the f32 path
    const void* src = a32 ? b : a;
    const int64_t span = a32 ? operand_span(batch, sBb, K, sBk, N, sBn) : operand_span(batch, sAb, M, sAm, K, sAk);
    void* wide = nullptr;
    if (int r = scratch.get_owned(4 * (size_t)span, st, &wide)) return r;
    if (!scratch.query) {
      const unsigned g = (unsigned)std::min<int64_t>((span + 255) / 256, 148 * 8);
      B200_LAUNCH(widen_bf16, dim3(g), dim3(256), 0, st, (const __nv_bfloat16*)src, (float*)wide, span);
    }
    return gemm_dispatch(a32 ? a : wide, a32 ? wide : b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb,
                         sBk, sBn, ldc, alpha, B200_DT_F32, out_dtype, epilogue, stream, scratch);
  }
  const int es = in_dtype == B200_DT_F32 ? 4 : 2;
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  auto m16 = [&](int64_t s) { return ((s * es) & 15) == 0; };
  int a_mn = -1, b_mn = -1;
  if (sAk == 1 && m16(sAm) && (batch == 1 || m16(sAb))) a_mn = 0;
  else if (sAm == 1 && m16(sAk) && (batch == 1 || m16(sAb))) a_mn = 1;
  if (sBk == 1 && m16(sBn) && (batch == 1 || m16(sBb))) b_mn = 0;
  else if (sBn == 1 && m16(sBk) && (batch == 1 || m16(sBb))) b_mn = 1;
  const bool tc = !force_simt() && a_mn >= 0 && b_mn >= 0 && al16(a) && al16(b) && K * es >= 16;
  const bool obf = out_dtype == B200_DT_BF16;
  if (tc) {
    const int64_t tiles128 = ((M + 127) / 128) * ((N + 127) / 128) * batch;
    const bool bn64 = N <= 64 || tiles128 < num_sms();
#define B200_TC(BN_, ES_, TO_, SPLIT_)                                                              \
  return launch_tc<BN_, ES_, TO_, SPLIT_>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, \
                                          ldc, alpha, epilogue, a_mn, b_mn, st, scratch)
    if (es == 4) {
      const bool x3 = f32_matmul_3x();
      if (x3 && use_persistent()) {
        // bf16 hi/lo planes on the persistent kernel (3 bf16 MMAs per step)
        int prc;
#define B200_PERS3(BN_, TO_)                                                                      \
  prc = launch_pers<BN_, TO_, 3>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, \
                                    ldc, alpha, epilogue, a_mn, b_mn, st, scratch)
        if (N <= 64) { if (obf) B200_PERS3(64, __nv_bfloat16); else B200_PERS3(64, float); }
        else if (N <= 128) { if (obf) B200_PERS3(128, __nv_bfloat16); else B200_PERS3(128, float); }
        else { if (obf) B200_PERS3(256, __nv_bfloat16); else B200_PERS3(256, float); }
#undef B200_PERS3
        if (prc != B200_ERR_UNSUPPORTED) return prc;
      }
      if (x3) {
        if (bn64) { if (obf) B200_TC(64, 4, __nv_bfloat16, true); else B200_TC(64, 4, float, true); }
        if (obf) B200_TC(128, 4, __nv_bfloat16, true); else B200_TC(128, 4, float, true);
      }
      if (bn64) { if (obf) B200_TC(64, 4, __nv_bfloat16, false); else B200_TC(64, 4, float, false); }
      if (obf) B200_TC(128, 4, __nv_bfloat16, false); else B200_TC(128, 4, float, false);
    } else {
      if (use_persistent()) {
        int prc;
#define B200_PERS(BN_, TO_)                                                                       \
  prc = launch_pers<BN_, TO_>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc,  \
                              alpha, epilogue, a_mn, b_mn, st, scratch)
        prc = B200_ERR_UNSUPPORTED;
        if (N > 128 && use_pair())
          prc = obf ? launch_pair<__nv_bfloat16>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk,
                                                 sBn, ldc, alpha, epilogue, a_mn, b_mn, st, scratch)
                    : launch_pair<float>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc,
                                         alpha, epilogue, a_mn, b_mn, st, scratch);
        if (prc != B200_ERR_UNSUPPORTED) return prc;
        if (N <= 64) { if (obf) B200_PERS(64, __nv_bfloat16); else B200_PERS(64, float); }
        else if (N <= 128) { if (obf) B200_PERS(128, __nv_bfloat16); else B200_PERS(128, float); }
        else { if (obf) B200_PERS(256, __nv_bfloat16); else B200_PERS(256, float); }
#undef B200_PERS
        if (prc != B200_ERR_UNSUPPORTED) return prc;
      }
      if (bn64) { if (obf) B200_TC(64, 2, __nv_bfloat16, false); else B200_TC(64, 2, float, false); }
      if (obf) B200_TC(128, 2, __nv_bfloat16, false); else B200_TC(128, 2, float, false);
    }
#undef B200_TC
  }
  if (es == 4) {
    if (obf) return launch_simt<float, __nv_bfloat16>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha, epilogue, st, scratch);
    return launch_simt<float, float>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha, epilogue, st, scratch);
  }
  if (obf) return launch_simt<__nv_bfloat16, __nv_bfloat16>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha, epilogue, st, scratch);
  return launch_simt<__nv_bfloat16, float>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha, epilogue, st, scratch);
}

}  // namespace
}  // namespace b200

namespace b200 {
namespace {
// A GEMM whose f32 operand(s) arrive as bf16 hi + lo planes (a_lo / b_lo not
// null; a / b then point at the hi planes).  in_dtype gives the logical types.
int gemm_planes_dispatch(const void* a, const void* a_lo, const void* b, const void* b_lo, void* c,
                         const void* bias, int64_t batch, int64_t M, int64_t N, int64_t K,
                         int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb, int64_t sBk,
                         int64_t sBn, int64_t ldc, float alpha, int in_dtype, int out_dtype,
                         int epilogue, void* stream, Scratch& scratch) {
  const bool a32 = in_dtype == B200_DT_F32 || in_dtype == B200_GEMM_DT_A_F32_B_BF16;
  const bool b32 = in_dtype == B200_DT_F32 || in_dtype == B200_GEMM_DT_A_BF16_B_F32;
  B200_CHECK_ARG((!a_lo || a32) && (!b_lo || b32), "gemm: planes given for a bf16 operand");
  B200_CHECK_ARG(a && b && c && batch >= 1 && M > 0 && N > 0 && K > 0, "gemm: bad planes call");
  if (ldc <= 0) ldc = N;
  auto st = (cudaStream_t)stream;
  const bool obf = out_dtype == B200_DT_BF16;
  auto m16 = [](int64_t s) { return ((s * 2) & 15) == 0; };
  int a_mn = -1, b_mn = -1;
  if (sAk == 1 && m16(sAm) && (batch == 1 || m16(sAb))) a_mn = 0;
  else if (sAm == 1 && m16(sAk) && (batch == 1 || m16(sAb))) a_mn = 1;
  if (sBk == 1 && m16(sBn) && (batch == 1 || m16(sBb))) b_mn = 0;
  else if (sBn == 1 && m16(sBk) && (batch == 1 || m16(sBb))) b_mn = 1;
  const int spl = (a32 ? 1 : 0) | (b32 ? 2 : 0);
  if (!force_simt() && use_persistent() && f32_matmul_3x() && a_mn >= 0 && b_mn >= 0 && spl) {
    int prc = B200_ERR_UNSUPPORTED;
#define B200_PERSP(BN_, TO_)                                                                        \
  prc = spl == 3 ? launch_pers<BN_, TO_, 3>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, \
                                            sBn, ldc, alpha, epilogue, a_mn, b_mn, st, scratch,     \
                                            a_lo, b_lo)                                             \
      : spl == 1 ? launch_pers<BN_, TO_, 1>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, \
                                            sBn, ldc, alpha, epilogue, a_mn, b_mn, st, scratch,     \
                                            a_lo, b_lo)                                             \
                 : launch_pers<BN_, TO_, 2>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, \
                                            sBn, ldc, alpha, epilogue, a_mn, b_mn, st, scratch,     \
                                            a_lo, b_lo)
    if (N <= 64) { if (obf) B200_PERSP(64, __nv_bfloat16); else B200_PERSP(64, float); }
    else if (N <= 128) { if (obf) B200_PERSP(128, __nv_bfloat16); else B200_PERSP(128, float); }
    else { if (obf) B200_PERSP(256, __nv_bfloat16); else B200_PERSP(256, float); }
#undef B200_PERSP
    if (prc != B200_ERR_UNSUPPORTED) return prc;
  }
  // otherwise: join the given planes back into f32 (x ~= hi + lo) and take the usual path
  void* wa = nullptr;
  void* wb = nullptr;
  const int64_t na = operand_span(batch, sAb, M, sAm, K, sAk), nb = operand_span(batch, sBb, K, sBk, N, sBn);
  if (a_lo) { if (int r = scratch.get_owned(4 * (size_t)na, st, &wa)) return r; }
  if (b_lo) { if (int r = scratch.get_owned(4 * (size_t)nb, st, &wb)) return r; }
  if (!scratch.query) {
    if (a_lo)
      B200_LAUNCH(join_planes, dim3((unsigned)std::min<int64_t>((na + 255) / 256, 148 * 8)), dim3(256), 0,
                  st, (const __nv_bfloat16*)a, (const __nv_bfloat16*)a_lo, (float*)wa, na);
    if (b_lo)
      B200_LAUNCH(join_planes, dim3((unsigned)std::min<int64_t>((nb + 255) / 256, 148 * 8)), dim3(256), 0,
                  st, (const __nv_bfloat16*)b, (const __nv_bfloat16*)b_lo, (float*)wb, nb);
  }
  return gemm_dispatch(a_lo ? wa : a, b_lo ? wb : b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk,
                       sBn, ldc, alpha, in_dtype, out_dtype, epilogue, stream, scratch);
}
}  // namespace
}  // namespace b200

extern "C" int64_t b200_gemm_planes_workspace_bytes(
    const void* a, const void* a_lo, const void* b, const void* b_lo, void* c, const void* bias,
    int64_t batch, int64_t M, int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk,
    int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, float alpha, int in_dtype, int out_dtype,
    int epilogue, void* stream) {
  b200::Scratch scratch;
  scratch.query = true;
  const int rc = b200::gemm_planes_dispatch(a, a_lo, b, b_lo, c, bias, batch, M, N, K, sAb, sAm, sAk,
                                            sBb, sBk, sBn, ldc, alpha, in_dtype, out_dtype, epilogue,
                                            stream, scratch);
  if (rc != b200::kWorkspaceQueried && rc != B200_OK) return -1;
  return (int64_t)scratch.queried;
}

extern "C" int b200_gemm_planes_ws(const void* a, const void* a_lo, const void* b, const void* b_lo,
                                   void* c, const void* bias, int64_t batch, int64_t M, int64_t N,
                                   int64_t K, int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
                                   int64_t sBk, int64_t sBn, int64_t ldc, float alpha, int in_dtype,
                                   int out_dtype, int epilogue, void* stream, void* ws,
                                   size_t ws_bytes) {
  b200::Scratch scratch;
  scratch.has_arena = true;
  scratch.arena = static_cast<uint8_t*>(ws);
  scratch.arena_bytes = ws ? ws_bytes : 0;
  return b200::gemm_planes_dispatch(a, a_lo, b, b_lo, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb,
                                    sBk, sBn, ldc, alpha, in_dtype, out_dtype, epilogue, stream,
                                    scratch);
}

extern "C" int b200_gemm(const void* a, const void* b, void* c, const void* bias, int64_t batch,
                         int64_t M, int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk,
                         int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, float alpha,
                         int in_dtype, int out_dtype, int epilogue, void* stream) {
  b200::Scratch scratch;  // split-K partials from cudaMallocAsync on `stream`
  return b200::gemm_dispatch(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc,
                             alpha, in_dtype, out_dtype, epilogue, stream, scratch);
}

// Workspace the call would take (split-K partials, bf16 planes of f32
// operands), without launching anything; the PJRT runtime hands it over from
// its caching allocator through b200_gemm_ws.  -1 on an argument error.
extern "C" int64_t b200_gemm_workspace_bytes(const void* a, const void* b, void* c, const void* bias,
                                             int64_t batch, int64_t M, int64_t N, int64_t K,
                                             int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
                                             int64_t sBk, int64_t sBn, int64_t ldc, float alpha,
                                             int in_dtype, int out_dtype, int epilogue, void* stream) {
  b200::Scratch scratch;
  scratch.query = true;
  const int rc = b200::gemm_dispatch(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn,
                                     ldc, alpha, in_dtype, out_dtype, epilogue, stream, scratch);
  if (rc != b200::kWorkspaceQueried && rc != B200_OK) return -1;
  return (int64_t)scratch.queried;
}

// b200_gemm taking its workspace from the caller (`ws`, `ws_bytes` from
// b200_gemm_workspace_bytes for the same arguments; may be null when that is 0).
extern "C" int b200_gemm_ws(const void* a, const void* b, void* c, const void* bias, int64_t batch,
                            int64_t M, int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk,
                            int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, float alpha,
                            int in_dtype, int out_dtype, int epilogue, void* stream, void* ws,
                            size_t ws_bytes) {
  b200::Scratch scratch;
  scratch.has_arena = true;
  scratch.arena = static_cast<uint8_t*>(ws);
  scratch.arena_bytes = ws ? ws_bytes : 0;
  return b200::gemm_dispatch(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc,
                             alpha, in_dtype, out_dtype, epilogue, stream, scratch);
}

// ---------------------------------------------------------------------------
// Allocation-free GEMM.  Split-K partial sums go to this fixed array instead of
// stream-ordered allocations, and the bounded-wait error word is a fixed
// device variable too, so a call never allocates device memory.  Every GPU
// that loads the library holds the array (kNoAllocScratchBytes) until the
// process exits; all calls on a device share it.
static constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];
static __device__ int g_noalloc_err;  // zero at load; set only by a wait that runs out

namespace b200 {
namespace {
struct NoAllocDevice {
  float* scratch = nullptr;
  int* err = nullptr;
};

// Device addresses of the fixed array and error word for the current device.
// In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory, so the address is looked up once per device (with that device
// current) and cached.
int noalloc_device(NoAllocDevice* out) {
  static std::mutex mu;
  static NoAllocDevice per[64];
  static bool ready[64] = {false};
  int dev = -1;
  B200_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(B200_ERR_INVALID, "gemm_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lk(mu);
  if (!ready[dev]) {
    B200_CUDA_TRY(cudaGetSymbolAddress((void**)&per[dev].scratch, g_noalloc_scratch));
    B200_CUDA_TRY(cudaGetSymbolAddress((void**)&per[dev].err, g_noalloc_err));
    ready[dev] = true;
  }
  *out = per[dev];
  return B200_OK;
}
}  // namespace

// Reads (and optionally clears) the allocation-free GEMM's error word on the
// current device; b200_device_error reports it together with its own word.
int noalloc_error_take(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_noalloc_err, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_noalloc_err, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}
}  // namespace b200

extern "C" int b200_gemm_noalloc(const void* a, const void* b, void* c, const void* bias,
                                 int64_t batch, int64_t M, int64_t N, int64_t K, int64_t sAb,
                                 int64_t sAm, int64_t sAk, int64_t sBb, int64_t sBk, int64_t sBn,
                                 int64_t ldc, float alpha, int in_dtype, int out_dtype,
                                 int epilogue, void* stream) {
  if (in_dtype != B200_DT_F32 && in_dtype != B200_DT_BF16)
    return b200::set_error(B200_ERR_UNSUPPORTED,
                           "gemm_noalloc: in_dtype must be F32 or BF16 (the mixed F32 x BF16 codes "
                           "need a widened or split copy of an operand, which this entry point "
                           "cannot allocate)");
  b200::NoAllocDevice nd;
  if (int rc = b200::noalloc_device(&nd)) return rc;
  b200::Scratch scratch;
  scratch.lent = nd.scratch;
  scratch.lent_bytes = kNoAllocScratchBytes;
  scratch.err = nd.err;
  return b200::gemm_dispatch(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc,
                             alpha, in_dtype, out_dtype, epilogue, stream, scratch);
}

// Which path b200_gemm takes for these arguments: 1 tensor cores, 0 SIMT.
extern "C" int b200_gemm_uses_tensor_cores(const void* a, const void* b, int64_t batch, int64_t K,
                                           int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
                                           int64_t sBk, int64_t sBn, int in_dtype) {
  const int es = in_dtype == B200_DT_F32 ? 4 : 2;
  auto m16 = [&](int64_t s) { return ((s * es) & 15) == 0; };
  const bool a_ok = (sAk == 1 && m16(sAm)) || (sAm == 1 && m16(sAk));
  const bool b_ok = (sBk == 1 && m16(sBn)) || (sBn == 1 && m16(sBk));
  const bool bat = batch == 1 || (m16(sAb) && m16(sBb));
  return !b200::force_simt() && a_ok && b_ok && bat && ((uintptr_t)a & 15) == 0 &&
         ((uintptr_t)b & 15) == 0 && K * es >= 16;
}
