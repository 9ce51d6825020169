// The cross-attention keys and values of every decoder layer from the encoder output, as one tcgen05 GEMM for
// sm_100a (the C ABI owsm_xkv_* of include/owsm_dec.h).
//
// Semantics: owsm-trt's Decoder.cross_kv (src/owsm_trt/modeling.py:490-499), which the sessions run once per
// utterance after the encoder (TorchBackend.encode, src/owsm_trt/runtime.py:63-74): for every layer l,
// K_l = enc W_k,l^T + b_k,l and V_l = enc W_v,l^T + b_v,l, split into heads -> cross_k / cross_v [L, U, H, T, 64].
//
// All layers are one GEMM: C[m, n] = sum_k enc[m, k] W[n, k] + b[n] with m = (utterance, frame) over U x T rows
// and n over the L x 2 x D rows of W = [W_k,0; W_v,0; W_k,1; ...] (fp16, packed at create). Tiles of 128 x 256
// outputs, K in steps of 64:
//   * warp 0 (one thread): TMA loads of the enc tile (128 x 64) and the W tile (256 x 64), 128-byte swizzle,
//     into a 4-stage shared-memory ring (48 KB a stage);
//   * warp 1: allocates 512 TMEM columns (two 256-column fp32 accumulators); one thread issues the
//     tcgen05.mma (M 128, N 256, K 16; four per stage) and commits each stage back to the producer and each
//     finished tile to the epilogue;
//   * warps 2-5: the epilogue, lane quarter (warp % 4) of the accumulator: 32 columns at a time from TMEM,
//     + bias, fp16, 64 contiguous bytes into the head's row of cross_k or cross_v. The next tile's MMAs run
//     into the other accumulator meanwhile.
// Persistent: one CTA per SM walks the tiles, M fastest (the CTAs working at one time share the W tile in L2).
// Every wait is bounded; a timed-out wait sets the handle's error word and the kernel runs to its end.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/owsm_dec.h"
#include "tc.cuh"

namespace owsm {

int record_error(int code, const std::string& msg);  // decoder.cu: the thread's last error message
static int fail(int code, const std::string& msg) { return record_error(code, msg); }

namespace xkv {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr uint32_t SPIN = 1u << 26;
constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 /* alignment */ + 256 /* barriers */;

struct Args {
  const float* bias;  // [N]
  __half* ck;         // [L][U][H][t_cap][64]
  __half* cv;
  int M, N, K;        // U * T rows, L * 2 * D columns, D
  int T, t_cap, U, H, D;
  int* err;
};

__device__ __forceinline__ void wait_or_flag(uint64_t* bar, uint32_t parity, int* err) {
  if (!mbar_wait(bar, parity, SPIN)) atomicExch(err, 1);
}

__global__ void __launch_bounds__(THREADS, 1)
xkv_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (a.M + BM - 1) / BM, tiles_n = a.N / BN, ntiles = tiles_m * tiles_n, nk = a.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // producer
      int s = 0;
      uint32_t ph = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const int m0 = (t % tiles_m) * BM, n0 = (t / tiles_m) * BN;
        for (int kb = 0; kb < nk; ++kb) {
          wait_or_flag(&empty[s], ph ^ 1u, a.err);
          uint8_t* sa = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(sa, &tm_a, kb * BK, m0, &full[s]);
          tma_load_2d(sa + A_BYTES, &tm_b, kb * BK, n0, &full[s]);
          if (++s == STAGES) s = 0, ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
      int s = 0;
      uint32_t ph = 0;
      int ab = 0;
      uint32_t aph = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        wait_or_flag(&acc_empty[ab], aph ^ 1u, a.err);  // the epilogue has read this accumulator out
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * BN);
        for (int kb = 0; kb < nk; ++kb) {
          wait_or_flag(&full[s], ph, a.err);
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES), sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_f16(d, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, (kb | kk) != 0);
          tc_commit(&empty[s]);  // the stage's slot is free once these MMAs have read it
          if (++s == STAGES) s = 0, ph ^= 1u;
        }
        tc_commit(&acc_full[ab]);
        if (++ab == 2) ab = 0, aph ^= 1u;
      }
    }
  } else {  // epilogue: warps 2..5 -> lane quarters 2, 3, 0, 1
    const int q = warp & 3;
    int ab = 0;
    uint32_t aph = 0;
    const int HD = a.H * 64;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const int m0 = (t % tiles_m) * BM, n0 = (t / tiles_m) * BN;
      wait_or_flag(&acc_full[ab], aph, a.err);
      tc_fence_after();
      const int m = m0 + q * 32 + lane;
      const int u = m / a.T, tt = m - u * a.T;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BN + c), r);
        tmem_ld_wait();
        if (m < a.M) {
          const int n = n0 + c, l = n / (2 * HD), rem = n - l * 2 * HD, kv = rem / HD, h = (rem - kv * HD) >> 6,
                    dd = rem & 63;
          __half* dst = (kv ? a.cv : a.ck) + ((((size_t)l * a.U + u) * a.H + h) * a.t_cap + tt) * 64 + dd;
          const float4* b4 = reinterpret_cast<const float4*>(a.bias + n);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 b0 = __ldg(b4 + 2 * j), b1 = __ldg(b4 + 2 * j + 1);
            uint4 o;
            o.x = pack_half2(__uint_as_float(r[8 * j + 0]) + b0.x, __uint_as_float(r[8 * j + 1]) + b0.y);
            o.y = pack_half2(__uint_as_float(r[8 * j + 2]) + b0.z, __uint_as_float(r[8 * j + 3]) + b0.w);
            o.z = pack_half2(__uint_as_float(r[8 * j + 4]) + b1.x, __uint_as_float(r[8 * j + 5]) + b1.y);
            o.w = pack_half2(__uint_as_float(r[8 * j + 6]) + b1.z, __uint_as_float(r[8 * j + 7]) + b1.w);
            reinterpret_cast<uint4*>(dst)[j] = o;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      if (++ab == 2) ab = 0, aph ^= 1u;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

__global__ void pack_rows_kernel(const void* __restrict__ src, int dtype, long long n, __half* __restrict__ dst) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = dtype == OWSM_DEC_F16 ? reinterpret_cast<const __half*>(src)[i]
                                   : __float2half_rn(reinterpret_cast<const float*>(src)[i]);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// A row-major fp16 matrix [rows][cols] as a 2D tensor map with boxes of 64 columns x box_rows rows, 128-byte swizzle.
int make_map(CUtensorMap* m, const void* base, long long rows, int cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(OWSM_DEC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OWSM_DEC_ERR_ARG, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return OWSM_DEC_OK;
}

}  // namespace xkv
}  // namespace owsm

using namespace owsm;

struct OwsmXkv {
  int device = 0, L = 0, D = 0, H = 0, N = 0, sms = 0;
  __half* w = nullptr;   // [N][D]
  float* b = nullptr;    // [N]
  int* err = nullptr;
  CUtensorMap tm_w;
};

#define XKV_TRY(x)                                                                               \
  do {                                                                                           \
    cudaError_t e_ = (x);                                                                        \
    if (e_ != cudaSuccess) return fail(OWSM_DEC_ERR_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

extern "C" {

int owsm_xkv_create(int L, int D, int H, int weight_dtype, const OwsmXkvLayer* layers, int device, OwsmXkv** out) {
  if (!layers || !out) return fail(OWSM_DEC_ERR_ARG, "null argument");
  *out = nullptr;
  if (L < 1 || H < 1 || D != H * 64 || D % xkv::BK) return fail(OWSM_DEC_ERR_LIMIT, "heads of 64 and D a multiple of 64");
  if ((L * 2 * D) % xkv::BN) return fail(OWSM_DEC_ERR_LIMIT, "L x 2D must be a multiple of 256");
  if (weight_dtype != OWSM_DEC_F32 && weight_dtype != OWSM_DEC_F16) return fail(OWSM_DEC_ERR_ARG, "weight dtype");
  int prev = 0;
  XKV_TRY(cudaGetDevice(&prev));
  XKV_TRY(cudaSetDevice(device));
  OwsmXkv* x = new OwsmXkv();
  x->device = device;
  x->L = L;
  x->D = D;
  x->H = H;
  x->N = L * 2 * D;
  auto bail = [&](int rc) {
    cudaFree(x->w);
    cudaFree(x->b);
    cudaFree(x->err);
    delete x;
    cudaSetDevice(prev);
    return rc;
  };
  int rc = OWSM_DEC_OK;
  if (cudaMalloc(&x->w, (size_t)x->N * D * 2) != cudaSuccess || cudaMalloc(&x->b, (size_t)x->N * 4) != cudaSuccess ||
      cudaMalloc(&x->err, 4) != cudaSuccess)
    return bail(fail(OWSM_DEC_ERR_CUDA, "cudaMalloc"));
  cudaMemset(x->err, 0, 4);
  for (int l = 0; l < L; ++l) {
    const void* w2[2] = {layers[l].wk, layers[l].wv};
    const float* b2[2] = {layers[l].bk, layers[l].bv};
    for (int kv = 0; kv < 2; ++kv) {
      if (!w2[kv] || !b2[kv]) return bail(fail(OWSM_DEC_ERR_ARG, "null K/V projection"));
      const size_t row0 = (size_t)(l * 2 + kv) * D;
      xkv::pack_rows_kernel<<<256, 256>>>(w2[kv], weight_dtype, (long long)D * D, x->w + row0 * D);
      if (cudaMemcpy(x->b + row0, b2[kv], (size_t)D * 4, cudaMemcpyDeviceToDevice) != cudaSuccess)
        return bail(fail(OWSM_DEC_ERR_CUDA, "bias copy"));
    }
  }
  if (cudaDeviceSynchronize() != cudaSuccess || cudaGetLastError() != cudaSuccess)
    return bail(fail(OWSM_DEC_ERR_CUDA, "packing the K/V projections"));
  if ((rc = xkv::make_map(&x->tm_w, x->w, x->N, D, xkv::BN))) return bail(rc);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return bail(fail(OWSM_DEC_ERR_CUDA, "properties"));
  if (prop.sharedMemPerBlockOptin < xkv::SMEM) return bail(fail(OWSM_DEC_ERR_LIMIT, "shared memory too small"));
  x->sms = prop.multiProcessorCount;
  if (cudaFuncSetAttribute(xkv::xkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)xkv::SMEM) != cudaSuccess)
    return bail(fail(OWSM_DEC_ERR_CUDA, "cudaFuncSetAttribute"));
  cudaSetDevice(prev);
  *out = x;
  return OWSM_DEC_OK;
}

int owsm_xkv_run(OwsmXkv* x, void* stream, const void* enc, int U, int T, int t_cap, void* cross_k, void* cross_v) {
  if (!x || !enc || !cross_k || !cross_v) return fail(OWSM_DEC_ERR_ARG, "null argument");
  if (U < 1 || T < 1 || t_cap < T) return fail(OWSM_DEC_ERR_ARG, "bad shape (U, T, t_cap)");
  if ((reinterpret_cast<uintptr_t>(enc) | reinterpret_cast<uintptr_t>(cross_k) | reinterpret_cast<uintptr_t>(cross_v)) & 127)
    return fail(OWSM_DEC_ERR_ARG, "enc, cross_k, cross_v must be 128-byte aligned");
  int prev = 0;
  XKV_TRY(cudaGetDevice(&prev));
  XKV_TRY(cudaSetDevice(x->device));
  CUtensorMap tm_a;
  const long long M = (long long)U * T;
  int rc = xkv::make_map(&tm_a, enc, M, x->D, xkv::BM);
  if (rc) {
    cudaSetDevice(prev);
    return rc;
  }
  xkv::Args a;
  a.bias = x->b;
  a.ck = reinterpret_cast<__half*>(cross_k);
  a.cv = reinterpret_cast<__half*>(cross_v);
  a.M = (int)M;
  a.N = x->N;
  a.K = x->D;
  a.T = T;
  a.t_cap = t_cap;
  a.U = U;
  a.H = x->H;
  a.D = x->D;
  a.err = x->err;
  const int ntiles = (int)((M + xkv::BM - 1) / xkv::BM) * (x->N / xkv::BN);
  const int grid = ntiles < x->sms ? ntiles : x->sms;
  xkv::xkv_kernel<<<grid, xkv::THREADS, xkv::SMEM, reinterpret_cast<cudaStream_t>(stream)>>>(tm_a, x->tm_w, a);
  const cudaError_t e = cudaGetLastError();
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(OWSM_DEC_ERR_CUDA, std::string("xkv launch: ") + cudaGetErrorString(e));
  return OWSM_DEC_OK;
}

int owsm_xkv_get_error(OwsmXkv* x) {
  if (!x) return fail(OWSM_DEC_ERR_ARG, "null handle");
  int prev = 0;
  XKV_TRY(cudaGetDevice(&prev));
  XKV_TRY(cudaSetDevice(x->device));
  int e = 0;
  const cudaError_t ce = cudaMemcpy(&e, x->err, 4, cudaMemcpyDeviceToHost);
  if (ce == cudaSuccess && e) cudaMemset(x->err, 0, 4);
  cudaSetDevice(prev);
  if (ce != cudaSuccess) return fail(OWSM_DEC_ERR_CUDA, cudaGetErrorString(ce));
  return e ? fail(OWSM_DEC_ERR_TIMEOUT, "a bounded wait of the K/V projection gave up") : OWSM_DEC_OK;
}

void owsm_xkv_destroy(OwsmXkv* x) {
  if (!x) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(x->device);
  cudaFree(x->w);
  cudaFree(x->b);
  cudaFree(x->err);
  cudaSetDevice(prev);
  delete x;
}

}  // extern "C"
