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
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "tc.cuh"

namespace b200 {
namespace {

constexpr int kStages = 4;

struct GemmArgs {
  int M, N, K;
  int a_mn, b_mn;
  float alpha;
  const void* bias;
  int epi;  // 0 none, 1 bias, 2 bias+relu, 3 relu
  void* c;
  int64_t ldc, sCb;
  int* err;
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

template <int BN, int ES, typename TO>
__global__ void __launch_bounds__(192, 1)
    gemm_tc(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
            GemmArgs p) {
  constexpr int BK = 128 / ES;  // K elements per 128-byte row
  constexpr int E = 128 / ES;   // MN elements per 128-byte chunk
  constexpr int A_BYTES = 128 * 128;
  constexpr int B_BYTES = BN * 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kStages * B_BYTES);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tfull + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * 128, bz = blockIdx.z;
  const int KB = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
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
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) + 1) & 1, abort, p.err, 101))
          break;
        mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
        if (!p.a_mn) {
          tma_load_3d(sA + s * A_BYTES, &tA, &full[s], kb * BK, m0, bz);
        } else {
#pragma unroll
          for (int i = 0; i < 128 / E; ++i)
            tma_load_3d(sA + s * A_BYTES + i * (BK * 128), &tA, &full[s], m0 + i * E, kb * BK, bz);
        }
        if (!p.b_mn) {
          tma_load_3d(sB + s * B_BYTES, &tB, &full[s], kb * BK, n0, bz);
        } else {
#pragma unroll
          for (int i = 0; i < BN / E; ++i)
            tma_load_3d(sB + s * B_BYTES + i * (BK * 128), &tB, &full[s], n0 + i * E, kb * BK, bz);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = umma_idesc(ES == 4 ? 2u : 1u, (uint32_t)p.a_mn, (uint32_t)p.b_mn, BN, 128);
      constexpr uint32_t KSTEP_MN = (32 / ES) * 128;  // bytes per MMA K-step, MN-major
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % kStages;
        if (!mbar_wait(&full[s], (kb / kStages) & 1, abort, p.err, 102)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * A_BYTES), b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = p.a_mn ? umma_desc(a0 + kk * KSTEP_MN, BK * 128, 1024)
                                     : umma_desc(a0 + kk * 32, 16, 1024);
          const uint64_t bd = p.b_mn ? umma_desc(b0 + kk * KSTEP_MN, BK * 128, 1024)
                                     : umma_desc(b0 + kk * 32, 16, 1024);
          if (ES == 4) umma_tf32(tmem, ad, bd, idesc, (kb | kk) != 0);
          else umma_f16(tmem, ad, bd, idesc, (kb | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(tfull);
    }
  } else {  // ---- epilogue: warps 2..5 drain TMEM lanes 32*(warp%4) ...
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int m = m0 + row;
    bool ok = mbar_wait(tfull, 0, abort, p.err, 103);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    if (ok) {
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

// SIMT fallback: 64x64 tile, 256 threads, 4x4 outputs per thread, f32 FMA.
template <typename TI, typename TO>
__global__ void __launch_bounds__(256)
    gemm_simt(const TI* __restrict__ A, const TI* __restrict__ B, TO* __restrict__ C,
              const void* bias, int M, int N, int K, int64_t sAb, int64_t sAm, int64_t sAk,
              int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, int64_t sCb, float alpha,
              int epi) {
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  const int bz = blockIdx.z;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  A += (int64_t)bz * sAb;
  B += (int64_t)bz * sBb;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int mm = i / 16, kk = i % 16;  // A tile [64 m][16 k]
      const int gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? Io<TI>::to_f(A[gm * sAm + gk * sAk]) : 0.f;
      const int kk2 = i / 64, nn = i % 64;  // B tile [16 k][64 n]
      const int gk2 = k0 + kk2, gn = n0 + nn;
      Bs[kk2][nn] = (gk2 < K && gn < N) ? Io<TI>::to_f(B[gk2 * sBk + gn * sBn]) : 0.f;
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
      float x = acc[i][j] * alpha;
      if (epi == 1 || epi == 2) x += Io<TO>::to_f(reinterpret_cast<const TO*>(bias)[n]);
      if (epi >= 2) x = fmaxf(x, 0.f);
      store_out<TO>(C + (int64_t)bz * sCb + (int64_t)m * ldc + n, x);
    }
  }
}

template <int BN, int ES, typename TO>
int launch_tc(const void* a, const void* b, void* c, const void* bias, int64_t batch, int64_t M,
              int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
              int64_t sBk, int64_t sBn, int64_t ldc, float alpha, int epi, int a_mn, int b_mn,
              cudaStream_t st) {
  constexpr int BK = 128 / ES;
  constexpr int E = 128 / ES;
  CUtensorMap ta, tb;
  int rc;
  if (!a_mn) {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sAm * ES), (uint64_t)(std::max<int64_t>(sAb, 1) * ES)};
    uint32_t box[3] = {(uint32_t)BK, 128, 1};
    rc = make_tmap(&ta, a, 3, dims, str, box, ES);
  } else {
    uint64_t dims[3] = {(uint64_t)M, (uint64_t)K, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sAk * ES), (uint64_t)(std::max<int64_t>(sAb, 1) * ES)};
    uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
    rc = make_tmap(&ta, a, 3, dims, str, box, ES);
  }
  if (rc) return rc;
  if (!b_mn) {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sBn * ES), (uint64_t)(std::max<int64_t>(sBb, 1) * ES)};
    uint32_t box[3] = {(uint32_t)BK, (uint32_t)BN, 1};
    rc = make_tmap(&tb, b, 3, dims, str, box, ES);
  } else {
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)batch};
    uint64_t str[2] = {(uint64_t)(sBk * ES), (uint64_t)(std::max<int64_t>(sBb, 1) * ES)};
    uint32_t box[3] = {(uint32_t)E, (uint32_t)BK, 1};
    rc = make_tmap(&tb, b, 3, dims, str, box, ES);
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
  p.err = device_error_word();
  if (!p.err) return set_error(B200_ERR_CUDA, "could not allocate the device error word");
  const int smem = kStages * (128 * 128 + BN * 128) + 1024 + 256;
  static bool attr = [&] {
    return cudaFuncSetAttribute(gemm_tc<BN, ES, TO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem) == cudaSuccess;
  }();
  if (!attr) return set_error(B200_ERR_CUDA, "cudaFuncSetAttribute(gemm_tc) failed");
  dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + 127) / 128), (unsigned)batch);
  gemm_tc<BN, ES, TO><<<grid, 192, smem, st>>>(ta, tb, p);
  B200_LAUNCH_CHECK();
  return B200_OK;
}

template <typename TI, typename TO>
int launch_simt(const void* a, const void* b, void* c, const void* bias, int64_t batch, int64_t M,
                int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk, int64_t sBb,
                int64_t sBk, int64_t sBn, int64_t ldc, float alpha, int epi, cudaStream_t st) {
  dim3 grid((unsigned)((N + 63) / 64), (unsigned)((M + 63) / 64), (unsigned)batch);
  gemm_simt<TI, TO><<<grid, 256, 0, st>>>((const TI*)a, (const TI*)b, (TO*)c, bias, (int)M, (int)N,
                                          (int)K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, M * ldc, alpha,
                                          epi);
  B200_LAUNCH_CHECK();
  return B200_OK;
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

extern "C" int b200_gemm(const void* a, const void* b, void* c, const void* bias, int64_t batch,
                         int64_t M, int64_t N, int64_t K, int64_t sAb, int64_t sAm, int64_t sAk,
                         int64_t sBb, int64_t sBk, int64_t sBn, int64_t ldc, float alpha,
                         int in_dtype, int out_dtype, int epilogue, void* stream) {
  using namespace b200;
  B200_CHECK_ARG(a && b && c, "gemm: null operand");
  B200_CHECK_ARG(batch >= 1 && M >= 0 && N >= 0 && K >= 0, "gemm: bad shape");
  B200_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31) && batch < 65536,
                 "gemm: dimension too large");
  B200_CHECK_ARG(epilogue >= 0 && epilogue <= 3, "gemm: bad epilogue");
  B200_CHECK_ARG(!(epilogue == 1 || epilogue == 2) || bias, "gemm: epilogue needs a bias");
  B200_CHECK_ARG(in_dtype == B200_DT_F32 || in_dtype == B200_DT_BF16, "gemm: in_dtype must be F32 or BF16");
  B200_CHECK_ARG(out_dtype == B200_DT_F32 || out_dtype == B200_DT_BF16, "gemm: out_dtype must be F32 or BF16");
  if (ldc <= 0) ldc = N;
  if (M == 0 || N == 0) return B200_OK;
  auto st = (cudaStream_t)stream;
  if (K == 0) return set_error(B200_ERR_UNSUPPORTED, "gemm: K == 0 is not supported");
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
#define B200_TC(BN_, ES_, TO_)                                                                      \
  return launch_tc<BN_, ES_, TO_>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, \
                                  alpha, epilogue, a_mn, b_mn, st)
    if (es == 4) {
      if (bn64) { if (obf) B200_TC(64, 4, __nv_bfloat16); else B200_TC(64, 4, float); }
      if (obf) B200_TC(128, 4, __nv_bfloat16); else B200_TC(128, 4, float);
    } else {
      if (bn64) { if (obf) B200_TC(64, 2, __nv_bfloat16); else B200_TC(64, 2, float); }
      if (obf) B200_TC(128, 2, __nv_bfloat16); else B200_TC(128, 2, float);
    }
#undef B200_TC
  }
  if (es == 4) {
    if (obf) return launch_simt<float, __nv_bfloat16>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha, epilogue, st);
    return launch_simt<float, float>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha, epilogue, st);
  }
  if (obf) return launch_simt<__nv_bfloat16, __nv_bfloat16>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha, epilogue, st);
  return launch_simt<__nv_bfloat16, float>(a, b, c, bias, batch, M, N, K, sAb, sAm, sAk, sBb, sBk, sBn, ldc, alpha, epilogue, st);
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
