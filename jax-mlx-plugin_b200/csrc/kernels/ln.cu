// Fused residual-add + LayerNorm / RMSNorm (forward and backward) for sm_100a.
//
// HBM-bound row kernels.  Forward: one warp per row; every lane keeps its share
// of the row in registers (16-byte vector loads, coalesced 512 B per warp
// instruction), so x and the residual are read once and y written once:
// 3*rows*cols*sizeof(T) bytes of traffic plus gamma/beta.  Mean and variance
// are two-pass in registers (no E[x^2]-E[x]^2 cancellation) with warp-shuffle
// sums.  Rows whose length does not fit the register path take a block-per-row
// kernel that re-reads the row from L1/L2.
//
// Math follows reference src/jax_mlx/layer_norm.py:20-25 (forward) and :59-76
// (backward); the residual add and affine are fused here where the reference
// ran them as separate MLX ops (src/jax_mlx_pjrt.cpp:4430-4437).
#include "common.cuh"

namespace b200 {
namespace {

// 4 rows (warps) per block: 1024 blocks for the 4096-row config, all resident at
// once (<= 64 registers -> 8 blocks per SM), so no second partial wave.
constexpr int kWarpsPerBlock = 4;

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* f);
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& u, float* f) {
  f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f);
template <>
__device__ __forceinline__ uint4 pack16<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}
template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 p = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&p);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Register-resident forward: NV 16-byte vectors per lane, cols = 32*NV*E.
template <typename T, int NV>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, NV <= 8 ? 8 : 4)
    ln_fwd_reg(const T* __restrict__ x, const T* __restrict__ res, const T* __restrict__ gamma,
               const T* __restrict__ beta, T* __restrict__ y, T* __restrict__ h,
               float* __restrict__ mean_out, float* __restrict__ rstd_out, int64_t rows,
               float eps, int kind) {
  pdl_wait();
  constexpr int E = 16 / sizeof(T);
  constexpr int COLS = 32 * NV * E;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * COLS;
  float v[NV * E];
  uint4 raw[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) raw[i] = ld_stream(xr + (i * 32 + lane) * E);
  if (res) {
    const T* rr = res + row * COLS;
    uint4 rraw[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) rraw[i] = ld_stream(rr + (i * 32 + lane) * E);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float a[E], b[E];
      unpack16<T>(raw[i], a);
      unpack16<T>(rraw[i], b);
#pragma unroll
      for (int e = 0; e < E; ++e) v[i * E + e] = a[e] + b[e];
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) unpack16<T>(raw[i], v + i * E);
  }
  if (h) {
    T* hr = h + row * COLS;
#pragma unroll
    for (int i = 0; i < NV; ++i) st_stream(hr + (i * 32 + lane) * E, pack16<T>(v + i * E));
  }
  const float inv_n = 1.0f / (float)COLS;
  float mean = 0.f;
  if (kind == 0) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NV * E; ++j) s += v[j];
    mean = warp_sum(s) * inv_n;
  }
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < NV * E; ++j) {
    const float d = v[j] - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(warp_sum(q) * inv_n + eps);
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
  T* yr = y + row * COLS;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = (i * 32 + lane) * E;
    float g[E], b[E], o[E];
    if (gamma) {
      unpack16<T>(*reinterpret_cast<const uint4*>(gamma + c), g);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) g[e] = 1.f;
    }
    if (beta) {
      unpack16<T>(*reinterpret_cast<const uint4*>(beta + c), b);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) b[e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = (v[i * E + e] - mean) * rstd * g[e] + b[e];
    st_stream(yr + c, pack16<T>(o));
  }
}

// Block-per-row forward for any cols: three passes over the row (L1/L2 hits
// after the first).
template <typename T>
__global__ void __launch_bounds__(256)
    ln_fwd_generic(const T* __restrict__ x, const T* __restrict__ res,
                   const T* __restrict__ gamma, const T* __restrict__ beta, T* __restrict__ y,
                   T* __restrict__ h, float* __restrict__ mean_out, float* __restrict__ rstd_out,
                   int64_t cols, float eps, int kind) {
  pdl_wait();
  __shared__ float red[32];
  __shared__ float stat;
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  const T* rr = res ? res + row * cols : nullptr;
  auto load = [&](int64_t c) {
    float a = Io<T>::to_f(xr[c]);
    if (rr) a += Io<T>::to_f(rr[c]);
    return a;
  };
  auto block_sum = [&](float s) {
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      t = warp_sum(t);
      if (threadIdx.x == 0) stat = t;
    }
    __syncthreads();
    const float r = stat;
    __syncthreads();
    return r;
  };
  float mean = 0.f;
  if (kind == 0) {
    float s = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) s += load(c);
    mean = block_sum(s) / (float)cols;
  }
  float q = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float d = load(c) - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(block_sum(q) / (float)cols + eps);
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = load(c);
    if (h) h[row * cols + c] = Io<T>::from_f(v);
    const float g = gamma ? Io<T>::to_f(gamma[c]) : 1.f;
    const float b = beta ? Io<T>::to_f(beta[c]) : 0.f;
    y[row * cols + c] = Io<T>::from_f((v - mean) * rstd * g + b);
  }
}

// Backward, one block per group of kBwdRowsPerBlock rows:
//   dx = rstd*(g*dy - mean(g*dy) - xhat*mean(g*dy*xhat)).
// Each block writes its partial column sums of dy*xhat and dy to
// ws[blockIdx.x][2][cols]; ln_bwd_colsum adds the partials up.
constexpr int kBwdRowsPerBlock = 16;

template <typename T>
__global__ void __launch_bounds__(256)
    ln_bwd_rows(const T* __restrict__ x, const T* __restrict__ gamma,
                const float* __restrict__ mean, const float* __restrict__ rstd,
                const T* __restrict__ dy, T* __restrict__ dx, float* __restrict__ ws,
                int64_t rows, int64_t cols) {
  pdl_wait();
  __shared__ float red[2][32];
  __shared__ float stat[2];
  const int64_t r0 = (int64_t)blockIdx.x * kBwdRowsPerBlock;
  const int64_t r1 = min(rows, r0 + kBwdRowsPerBlock);
  float* pg = ws + (int64_t)blockIdx.x * 2 * cols;  // partial dgamma
  float* pb = pg + cols;                             // partial dbeta
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) { pg[c] = 0.f; pb[c] = 0.f; }
  for (int64_t r = r0; r < r1; ++r) {
    const float mu = mean[r], rs = rstd[r];
    float s1 = 0.f, s2 = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const float xh = (Io<T>::to_f(x[r * cols + c]) - mu) * rs;
      const float g = gamma ? Io<T>::to_f(gamma[c]) : 1.f;
      const float d = Io<T>::to_f(dy[r * cols + c]);
      s1 += g * d;
      s2 += g * d * xh;
      pg[c] += d * xh;
      pb[c] += d;
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if ((threadIdx.x & 31) == 0) { red[0][threadIdx.x >> 5] = s1; red[1][threadIdx.x >> 5] = s2; }
    __syncthreads();
    if (threadIdx.x < 32) {
      const bool ok = threadIdx.x < (blockDim.x >> 5);
      float a = warp_sum(ok ? red[0][threadIdx.x] : 0.f);
      float b = warp_sum(ok ? red[1][threadIdx.x] : 0.f);
      if (threadIdx.x == 0) { stat[0] = a; stat[1] = b; }
    }
    __syncthreads();
    const float m1 = stat[0] / (float)cols, m2 = stat[1] / (float)cols;
    __syncthreads();
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const float xh = (Io<T>::to_f(x[r * cols + c]) - mu) * rs;
      const float g = gamma ? Io<T>::to_f(gamma[c]) : 1.f;
      const float d = Io<T>::to_f(dy[r * cols + c]);
      dx[r * cols + c] = Io<T>::from_f(rs * (g * d - m1 - xh * m2));
    }
  }
}

__global__ void ln_bwd_colsum(const float* __restrict__ ws, float* __restrict__ dgamma,
                              float* __restrict__ dbeta, int64_t nblk, int64_t cols) {
  pdl_wait();
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float g = 0.f, b = 0.f;
  for (int64_t i = 0; i < nblk; ++i) {
    g += ws[i * 2 * cols + c];
    b += ws[i * 2 * cols + cols + c];
  }
  if (dgamma) dgamma[c] = g;
  if (dbeta) dbeta[c] = b;
}

template <typename T>
int launch_fwd(const void* x, const void* res, const void* gamma, const void* beta, void* y,
               void* h, float* mean_out, float* rstd_out, int64_t rows, int64_t cols, float eps,
               int kind, cudaStream_t st) {
  constexpr int E = 16 / sizeof(T);
  const bool aligned = ((uintptr_t)x % 16 == 0) && (!res || (uintptr_t)res % 16 == 0) &&
                       ((uintptr_t)y % 16 == 0) && (!h || (uintptr_t)h % 16 == 0) &&
                       (!gamma || (uintptr_t)gamma % 16 == 0) && (!beta || (uintptr_t)beta % 16 == 0);
  const int64_t nv = cols / (32 * E);
  const dim3 grid((unsigned)((rows + kWarpsPerBlock - 1) / kWarpsPerBlock));
  const dim3 block(kWarpsPerBlock * 32);
  auto X = (const T*)x; auto R = (const T*)res; auto G = (const T*)gamma; auto B = (const T*)beta;
  auto Y = (T*)y; auto H = (T*)h;
  if (aligned && cols == nv * 32 * E) {
    switch (nv) {
#define B200_LN_CASE(n) \
  case n: B200_LAUNCH(ln_fwd_reg<T, n>, grid, block, 0, st, X, R, G, B, Y, H, mean_out, rstd_out, rows, eps, kind); return B200_OK;
      B200_LN_CASE(1) B200_LN_CASE(2) B200_LN_CASE(3) B200_LN_CASE(4) B200_LN_CASE(5)
      B200_LN_CASE(6) B200_LN_CASE(7) B200_LN_CASE(8) B200_LN_CASE(12) B200_LN_CASE(16)
#undef B200_LN_CASE
      default: break;
    }
  }
  B200_LAUNCH(ln_fwd_generic<T>, dim3((unsigned)rows), dim3(256), 0, st, X, R, G, B, Y, H,
              mean_out, rstd_out, cols, eps, kind);
  return B200_OK;
}

template <typename T>
int launch_bwd(const void* x, const void* gamma, const float* mean, const float* rstd,
               const void* dy, void* dx, float* dgamma, float* dbeta, void* ws, int64_t rows,
               int64_t cols, cudaStream_t st) {
  const int64_t nblk = (rows + kBwdRowsPerBlock - 1) / kBwdRowsPerBlock;
  B200_LAUNCH(ln_bwd_rows<T>, dim3((unsigned)nblk), dim3(256), 0, st, (const T*)x,
              (const T*)gamma, mean, rstd, (const T*)dy, (T*)dx, (float*)ws, rows, cols);
  B200_LAUNCH(ln_bwd_colsum, dim3((unsigned)((cols + 255) / 256)), dim3(256), 0, st,
              (const float*)ws, dgamma, dbeta, nblk, cols);
  return B200_OK;
}

}  // namespace
}  // namespace b200

extern "C" int b200_ln_residual_fwd(const void* x, const void* residual, const void* gamma,
                                    const void* beta, void* y, void* h_out, float* mean_out,
                                    float* rstd_out, int64_t rows, int64_t cols, float eps,
                                    int dtype, int kind, void* stream) {
  B200_CHECK_ARG(x && y, "ln_residual_fwd: x and y are required");
  B200_CHECK_ARG(rows >= 0 && cols > 0, "ln_residual_fwd: bad shape");
  B200_CHECK_ARG(kind == 0 || kind == 1, "ln_residual_fwd: kind must be 0 (LN) or 1 (RMS)");
  B200_CHECK_ARG(rows < (1ll << 31), "ln_residual_fwd: too many rows");
  if (rows == 0) return B200_OK;
  auto st = (cudaStream_t)stream;
  if (dtype == B200_DT_F32)
    return b200::launch_fwd<float>(x, residual, gamma, beta, y, h_out, mean_out, rstd_out, rows,
                                   cols, eps, kind, st);
  if (dtype == B200_DT_BF16)
    return b200::launch_fwd<__nv_bfloat16>(x, residual, gamma, beta, y, h_out, mean_out, rstd_out,
                                           rows, cols, eps, kind, st);
  return b200::set_error(B200_ERR_UNSUPPORTED, "ln_residual_fwd: dtype must be F32 or BF16");
}

extern "C" int64_t b200_ln_bwd_workspace(int64_t rows, int64_t cols) {
  const int64_t nblk = (rows + b200::kBwdRowsPerBlock - 1) / b200::kBwdRowsPerBlock;
  return nblk * 2 * cols * (int64_t)sizeof(float);
}

extern "C" int b200_ln_bwd(const void* x, const void* gamma, const float* mean, const float* rstd,
                           const void* dy, void* dx, float* dgamma, float* dbeta, void* ws,
                           int64_t rows, int64_t cols, int dtype, void* stream) {
  B200_CHECK_ARG(x && mean && rstd && dy && dx && ws, "ln_bwd: null argument");
  B200_CHECK_ARG(rows > 0 && cols > 0 && rows < (1ll << 31), "ln_bwd: bad shape");
  auto st = (cudaStream_t)stream;
  if (dtype == B200_DT_F32)
    return b200::launch_bwd<float>(x, gamma, mean, rstd, dy, dx, dgamma, dbeta, ws, rows, cols, st);
  if (dtype == B200_DT_BF16)
    return b200::launch_bwd<__nv_bfloat16>(x, gamma, mean, rstd, dy, dx, dgamma, dbeta, ws, rows,
                                           cols, st);
  return b200::set_error(B200_ERR_UNSUPPORTED, "ln_bwd: dtype must be F32 or BF16");
}
