// fk_paged_append.cu -- write one new token's K and V per sequence into a
// paged KV pool (16-token pages), optionally quantising to e4m3 on the way.
//
// Replaces the reference's Python per-token loop
// (fskernels/paged_attn/paged_kv_cache.py:109-132, driven per sequence and
// per layer by benchmarks/run_hf_triton_fp8_paged.py:38-43), which reads the
// block table back to the host for every token, and the per-step whole-cache
// quantize_to_fp8 of the FP8 adapter (triton_gqa_decode_hf_fp8.py:268-269).
// Positions come from a device array, so a decode step (append + attention)
// can be captured in a CUDA graph; page allocation stays on the host.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/fk_decode.h"

namespace fk {
int fail(int code, const char* fmt, ...);

struct AppendParams {
  const void* k_new;
  const void* v_new;
  long long kn_b, kn_h, vn_b, vn_h;  // element strides of k_new / v_new [B, KVH, D]
  void* k_pool;
  void* v_pool;
  long long kp_p, kp_h, kp_s, vp_p, vp_h, vp_s;  // element strides of the pools
  const int* bt;
  long long bt_b;
  int max_blocks;
  long long num_pages;
  int* pos;           // [B] write position of each sequence (its current length)
  int increment;      // add 1 to pos[b] after writing
  const float* scale_k;
  const float* scale_v;
  int* status;        // optional FK_STATUS_* word
  int B, kvh, in_dtype, pool_dtype;
  int head_dim;       // 128, or 64
};

__device__ __forceinline__ float load_elem(const void* base, long long i, int dt) {
  if (dt == FK_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
  return __half2float(static_cast<const __half*>(base)[i]);
}

// One CTA per sequence; with tph = D / 8 threads per head, thread t handles
// dims 8*(t%tph) .. +7 of KV head t/tph (and further heads in steps of
// blockDim/tph).
__global__ void __launch_bounds__(128) paged_append_kernel(const AppendParams p) {
  const int b = blockIdx.x;
  const int pos = p.pos[b];
  __syncthreads();  // every thread has read pos before thread 0 may bump it
  const int page = pos >> 4, slot = pos & 15;
  const int phys = (pos >= 0 && page < p.max_blocks) ? p.bt[static_cast<long long>(b) * p.bt_b + page] : -1;
  if (phys < 0 || phys >= p.num_pages) {
    if (threadIdx.x == 0 && p.status != nullptr) atomicOr(p.status, FK_STATUS_BAD_PAGE);
    return;
  }
  // x / scale, as the reference's quantize_to_fp8 computes it (a true
  // division: multiplying by a reciprocal would round differently)
  const float sk = (p.scale_k != nullptr) ? __ldg(p.scale_k) : 1.f;
  const float sv = (p.scale_v != nullptr) ? __ldg(p.scale_v) : 1.f;
  const int tph = p.head_dim / 8;
  const int d0 = (threadIdx.x % tph) * 8;
  for (int h = threadIdx.x / tph; h < p.kvh; h += blockDim.x / tph) {
    const long long ki = static_cast<long long>(b) * p.kn_b + static_cast<long long>(h) * p.kn_h + d0;
    const long long vi = static_cast<long long>(b) * p.vn_b + static_cast<long long>(h) * p.vn_h + d0;
    const long long ko = static_cast<long long>(phys) * p.kp_p + static_cast<long long>(h) * p.kp_h +
                         static_cast<long long>(slot) * p.kp_s + d0;
    const long long vo = static_cast<long long>(phys) * p.vp_p + static_cast<long long>(h) * p.vp_h +
                         static_cast<long long>(slot) * p.vp_s + d0;
    if (p.pool_dtype == FK_DTYPE_E4M3) {
      // x / scale, saturated to +-448, rounded to nearest e4m3
      uint32_t kw[2], vw[2];
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        uint32_t kk = 0, vv = 0;
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const float2 kx = make_float2(load_elem(p.k_new, ki + 4 * w + e, p.in_dtype) / sk,
                                        load_elem(p.k_new, ki + 4 * w + e + 1, p.in_dtype) / sk);
          const float2 vx = make_float2(load_elem(p.v_new, vi + 4 * w + e, p.in_dtype) / sv,
                                        load_elem(p.v_new, vi + 4 * w + e + 1, p.in_dtype) / sv);
          kk |= static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(kx, __NV_SATFINITE, __NV_E4M3)) << (8 * e);
          vv |= static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(vx, __NV_SATFINITE, __NV_E4M3)) << (8 * e);
        }
        kw[w] = kk;
        vw[w] = vv;
      }
      *reinterpret_cast<uint2*>(static_cast<unsigned char*>(p.k_pool) + ko) = make_uint2(kw[0], kw[1]);
      *reinterpret_cast<uint2*>(static_cast<unsigned char*>(p.v_pool) + vo) = make_uint2(vw[0], vw[1]);
    } else {
      // same 16-bit type: a straight 16-byte copy
      *reinterpret_cast<uint4*>(static_cast<unsigned short*>(p.k_pool) + ko) =
          *reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(p.k_new) + ki);
      *reinterpret_cast<uint4*>(static_cast<unsigned short*>(p.v_pool) + vo) =
          *reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(p.v_new) + vi);
    }
  }
  if (p.increment && threadIdx.x == 0) p.pos[b] = pos + 1;
}

}  // namespace fk

using namespace fk;

extern "C" int fk_paged_kv_append(const void* k_new, const void* v_new, int in_dtype, void* k_pool, void* v_pool,
                                  int pool_dtype, const int32_t* block_table, int32_t* positions, int increment,
                                  const float* scale_k, const float* scale_v, int* status, int batch, int kv_heads,
                                  int head_dim, int64_t num_pages, int max_blocks, int64_t skn_b, int64_t skn_h,
                                  int64_t svn_b, int64_t svn_h, int64_t sk_p, int64_t sk_h, int64_t sk_s,
                                  int64_t sv_p, int64_t sv_h, int64_t sv_s, int64_t bt_b, void* stream) {
  if (batch == 0) return FK_OK;
  if (k_new == nullptr || v_new == nullptr || k_pool == nullptr || v_pool == nullptr || block_table == nullptr ||
      positions == nullptr)
    return fail(FK_ERR_INVALID_ARG, "k_new, v_new, pools, block_table and positions must be non-null");
  if (batch < 0 || kv_heads <= 0 || num_pages <= 0 || max_blocks < 0)
    return fail(FK_ERR_INVALID_ARG, "bad sizes");
  if (head_dim != 128 && head_dim != 64) return fail(FK_ERR_UNSUPPORTED, "head_dim must be 128 or 64 (got %d)", head_dim);
  if (in_dtype != FK_DTYPE_F16 && in_dtype != FK_DTYPE_BF16)
    return fail(FK_ERR_UNSUPPORTED, "new K/V must be f16 or bf16");
  if (pool_dtype != FK_DTYPE_E4M3 && pool_dtype != in_dtype)
    return fail(FK_ERR_INVALID_ARG, "a 16-bit pool must have the dtype of the new K/V");
  const int es = (pool_dtype == FK_DTYPE_E4M3) ? 1 : 2;
  if (((sk_p | sk_h | sk_s | sv_p | sv_h | sv_s) * es) % 16 != 0 || ((skn_b | skn_h | svn_b | svn_h) * 2) % 16 != 0)
    return fail(FK_ERR_INVALID_ARG, "strides must be multiples of 16 bytes");
  if (((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
        reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool)) & 15) != 0)
    return fail(FK_ERR_INVALID_ARG, "tensors must be 16-byte aligned");
  AppendParams p{};
  p.k_new = k_new;
  p.v_new = v_new;
  p.kn_b = skn_b;
  p.kn_h = skn_h;
  p.vn_b = svn_b;
  p.vn_h = svn_h;
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.kp_p = sk_p;
  p.kp_h = sk_h;
  p.kp_s = sk_s;
  p.vp_p = sv_p;
  p.vp_h = sv_h;
  p.vp_s = sv_s;
  p.bt = block_table;
  p.bt_b = bt_b;
  p.max_blocks = max_blocks;
  p.num_pages = num_pages;
  p.pos = positions;
  p.increment = increment;
  p.scale_k = scale_k;
  p.scale_v = scale_v;
  p.status = status;
  p.B = batch;
  p.kvh = kv_heads;
  p.in_dtype = in_dtype;
  p.pool_dtype = pool_dtype;
  p.head_dim = head_dim;
  paged_append_kernel<<<batch, 128, 0, static_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FK_ERR_CUDA, "paged append launch failed: %s", cudaGetErrorString(e));
  return FK_OK;
}
