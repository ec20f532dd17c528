// fk_decode.cu -- host side of the B200 (sm_100a) GQA decode attention
// library: grid sizing, tensor maps, launch, and the C-ABI declared in
// include/fk_decode.h.  The kernel and the design notes are in
// fk_decode_kernel.cuh.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "fk_decode_kernel.cuh"

// The kernels are instantiated in fk_kernels_{f16,bf16,e4m3}.cu; a build of
// this file alone (e.g. the -DFK_TRACE diagnostics build) defines
// FK_SINGLE_TU and instantiates them here.
#ifndef FK_SINGLE_TU
FK_KERNELS_F16(FK_KERNEL_DECL)
FK_KERNELS_BF16(FK_KERNEL_DECL)
FK_KERNELS_E4M3(FK_KERNEL_DECL)
#endif

namespace fk {

// ------------------------------------------------------------------------
// Host side.
// ------------------------------------------------------------------------
thread_local std::string g_err;

// Optional per-launch timing: when enabled, events are recorded on the
// launching stream just before and just after each decode kernel.
struct Profiler {
  std::mutex mu;
  bool on = false;
  int cap = 0, n = 0;
  cudaEvent_t* ev = nullptr;  // 2 per launch
};
Profiler g_prof;

void prof_mark(int which, cudaStream_t stream) {
  if (!g_prof.on) return;
  std::lock_guard<std::mutex> lk(g_prof.mu);
  if (!g_prof.on || g_prof.n >= g_prof.cap) return;
  cudaEventRecord(g_prof.ev[2 * g_prof.n + which], stream);
  if (which == 1) ++g_prof.n;
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

template <int KV, int HP, int D, bool CP>
constexpr size_t smem_bytes() {
  using C = KvCfg<KV, D, CP>;
  return 1024 + C::STAGES * (C::STAGE_BYTES + sizeof(Meta) + 2 * sizeof(uint64_t)) +
         C::QSLOTS * (sizeof(uint32_t) * HP * GPAD * 64 + sizeof(uint64_t)) +
         C::NSLOT * (sizeof(EpiSlot) + sizeof(Meta) + 2 * sizeof(uint64_t));
}

// Query chunks per KV head: groups of more than 8 query heads are split into
// items of at most 8 (the MMA N), each reading its KV head.
inline int qc_for(int q_heads, int kv_heads) {
  const int g = (kv_heads > 0) ? q_heads / kv_heads : 1;
  return g > 8 ? (g + 7) / 8 : 1;
}

// KV heads per work item: 2 when kv_heads is even (one TMA box then covers
// both heads of a page) and the group fits one item, else 1; e4m3 KV with
// kv_heads % 4 == 0, a group of 5..8 query heads and 16-byte-aligned Q rows
// takes 4 (one 8 KB box per page and head quad: half the TMA issues per
// byte).  Measured: config 5 (G = 8, paged) 1.4-2.5 % faster with 4;
// config 4 (G = 4, paged) and its dense cache 2-5 % slower, so groups of at
// most 4 keep 2.
// FK_DECODE_HP=1 / =2 in the environment caps the heads per item (a tuning
// knob; read once, applies to every layout so paged and contiguous results
// stay bit-identical).
inline int hp_for(int kv_heads, int qc = 1, int kv = -1, int q_al16 = 0, int group = 8) {
  static const int cap = [] {
    const char* e = getenv("FK_DECODE_HP");
    return (e != nullptr && (e[0] == '1' || e[0] == '2')) ? e[0] - '0' : 4;
  }();
  if (cap == 1) return 1;
  if (qc > 1) return 2;  // chunk pairs of one KV head
  if (cap >= 4 && kv == FK_DTYPE_E4M3 && q_al16 && kv_heads % 4 == 0 && group > 4) return 4;
  return (kv_heads % 2 == 0) ? 2 : 1;
}

// Grid sizes a workspace is planned for: four-head items use two 16-slot
// records per segment, so their layout is planned for twice the CTAs.
inline int ws_ctas(int S, int hp) { return hp == 4 ? 2 * S : S; }

// Rows per pipeline stage (tokens x item heads) of the kernel for (kv, D).
inline uint32_t tile_rows(int kv, int head_dim) {
  return (kv != FK_DTYPE_E4M3 && head_dim == 64) ? 128u : 64u;
}

// KV heads in one TMA box: chunk pairs load a single head.
inline uint32_t box_heads(int hp, int qc) { return static_cast<uint32_t>((qc > 1) ? 1 : hp); }

template <int KV, int LAYOUT, int HP, int D, bool CP, bool QC>
int prepare_kernel(int device) {
  static bool done[64] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (device < 0 || device >= 64) return fail(FK_ERR_INVALID_ARG, "device index %d out of range", device);
  if (!done[device]) {
    cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<KV, LAYOUT, HP, D, CP, QC>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem_bytes<KV, HP, D, CP>()));
    if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    done[device] = true;
  }
  return FK_OK;
}

template <int KV, int HP, int D, bool CP>
int occupancy(int device, int* per_sm) {
  int rc = prepare_kernel<KV, VARLEN, HP, D, CP, false>(device);
  if (rc != FK_OK) return rc;
  const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      per_sm, decode_split_kernel<KV, VARLEN, HP, D, CP, false>, THREADS, smem_bytes<KV, HP, D, CP>());
  return e == cudaSuccess ? FK_OK : fail(FK_ERR_CUDA, "occupancy query failed: %s", cudaGetErrorString(e));
}

// Resident CTAs of the decode kernel on `device` for KV type `kv`, HP KV
// heads per item and head dim d: the persistent grid size S.  It does not
// depend on the layout (the layout instantiations share shared-memory
// footprint and launch bounds), so paged, dense and varlen calls plan
// identical segments.
int num_work_ctas(int device, int kv, int hp, int d = HEAD_DIM, bool cp = false) {
  static int cache[64][3][4][2][2] = {};
  static std::mutex mu;
  if (device < 0 || device >= 64 || kv < 0 || kv > 2 || hp < 1 || hp > 4 || hp == 3 || (cp && hp != 2)) return 0;
  if (hp == 4 && kv != FK_DTYPE_E4M3) return 0;
  if (d != 128 && (d != 64 || kv == FK_DTYPE_E4M3)) return 0;
  const int di = d == 64 ? 0 : 1, ci = cp ? 1 : 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (cache[device][kv][hp - 1][di][ci] > 0) return cache[device][kv][hp - 1][di][ci];
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  int per_sm = 0, prev = 0;
  cudaGetDevice(&prev);
  if (prev != device) cudaSetDevice(device);
#define FK_OCC(KVT, H, DD, CC) occupancy<KVT, H, DD, CC>(device, &per_sm)
#define FK_OCC_D(KVT, DD) (cp ? FK_OCC(KVT, 2, DD, true) : hp == 2 ? FK_OCC(KVT, 2, DD, false) : FK_OCC(KVT, 1, DD, false))
  int rc;
  if (kv == FK_DTYPE_F16) rc = d == 64 ? FK_OCC_D(FK_DTYPE_F16, 64) : FK_OCC_D(FK_DTYPE_F16, 128);
  else if (kv == FK_DTYPE_BF16) rc = d == 64 ? FK_OCC_D(FK_DTYPE_BF16, 64) : FK_OCC_D(FK_DTYPE_BF16, 128);
  else rc = hp == 4 ? FK_OCC(FK_DTYPE_E4M3, 4, 128, false) : FK_OCC_D(FK_DTYPE_E4M3, 128);
#undef FK_OCC_D
#undef FK_OCC
  if (prev != device) cudaSetDevice(prev);
  if (rc != FK_OK || per_sm <= 0) return 0;
  std::lock_guard<std::mutex> lk(mu);
  cache[device][kv][hp - 1][di][ci] = sms * per_sm;
  return cache[device][kv][hp - 1][di][ci];
}

// Grid size a workspace must be planned for: the largest over the head dims
// the KV type supports (the workspace size functions do not take the head
// dim), with chunk pairs when the group needs them.
int num_work_ctas_any_d(int device, int kv, int hp, bool cp) {
  const int s128 = num_work_ctas(device, kv, hp, 128, cp);
  const int s64 = (kv == FK_DTYPE_E4M3) ? 0 : num_work_ctas(device, kv, hp, 64, cp);
  return (s128 <= 0 || (kv != FK_DTYPE_E4M3 && s64 <= 0)) ? 0 : (s128 > s64 ? s128 : s64);
}

int encode_map(CUtensorMap* map, int kv, int rank, const void* base, const uint64_t* dims, const uint64_t* strides_b,
               const uint32_t* box) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(FK_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t gd[5];
  cuuint64_t gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_b[i];
  const CUtensorMapDataType dt = (kv == FK_DTYPE_E4M3)   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : (kv == FK_DTYPE_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, rank, const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FK_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return FK_OK;
}

bool is16(int dt) { return dt == FK_DTYPE_F16 || dt == FK_DTYPE_BF16; }

int common_checks(const void* q, const void* k, const void* v, const void* out, int batch, int q_heads, int kv_heads,
                  int head_dim, int q_dtype, int kv_dtype, int out_dtype, void* ws, int* device) {
  if (batch == 0) return FK_EMPTY;  // nothing to do; pointers of empty tensors may be null
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(FK_ERR_INVALID_ARG, "q, k, v and out must be non-null");
  if (ws == nullptr) return fail(FK_ERR_WORKSPACE, "workspace must be non-null");
  if (batch < 0 || q_heads <= 0 || kv_heads <= 0)
    return fail(FK_ERR_INVALID_ARG, "bad sizes: batch=%d q_heads=%d kv_heads=%d", batch, q_heads, kv_heads);
  if (head_dim != 128 && !(head_dim == 64 && kv_dtype != FK_DTYPE_E4M3))
    return fail(FK_ERR_UNSUPPORTED, "head_dim must be 128, or 64 with f16/bf16 KV (got %d)", head_dim);
  if (q_heads % kv_heads != 0)
    return fail(FK_ERR_INVALID_ARG, "q_heads (%d) must be a multiple of kv_heads (%d)", q_heads, kv_heads);
  if (!is16(out_dtype)) return fail(FK_ERR_UNSUPPORTED, "out dtype must be f16 or bf16");
  if (kv_dtype != FK_DTYPE_E4M3 && !is16(kv_dtype)) return fail(FK_ERR_UNSUPPORTED, "unsupported kv dtype %d", kv_dtype);
  if (q_dtype != FK_DTYPE_E4M3 && !is16(q_dtype)) return fail(FK_ERR_UNSUPPORTED, "unsupported q dtype %d", q_dtype);
  if (is16(kv_dtype) && q_dtype != kv_dtype)
    return fail(FK_ERR_INVALID_ARG, "q dtype must equal the 16-bit kv dtype");
  const int es = (kv_dtype == FK_DTYPE_E4M3) ? 1 : 2;
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15)
    return fail(FK_ERR_INVALID_ARG, "k/v base addresses must be 16-byte aligned");
  (void)es;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, k) != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return fail(FK_ERR_INVALID_ARG, "k must be device memory");
  }
  *device = attr.device;
  return FK_OK;
}

// Diagnostics set through fk_debug_configure: the bound of every mbarrier
// wait and the stage-withholding test hook (see Params::inject).
std::atomic<unsigned long long> g_wait_ns{4000000000ull};
std::atomic<int> g_inject{0};

// Programmatic dependent launch (default on; FK_DECODE_PDL=0 turns it off):
// the decode grid may be scheduled while the previous kernel of its stream
// drains, and executes griddepcontrol.wait before its first global read, so
// whatever that kernel wrote (KV append, RoPE'd Q, new lengths) is visible.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("FK_DECODE_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

template <int KV, int LAYOUT, int HP, int D, bool CP, bool QC>
int launch_one(const Params& p, int S, int device, cudaStream_t stream) {
  const int rc = prepare_kernel<KV, LAYOUT, HP, D, CP, QC>(device);
  if (rc != FK_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem_bytes<KV, HP, D, CP>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_split_kernel<KV, LAYOUT, HP, D, CP, QC>, p);
  if (e != cudaSuccess) return fail(FK_ERR_CUDA, "cudaLaunchKernelEx: %s", cudaGetErrorString(e));
  return FK_OK;
}

template <int LAYOUT>
int launch(Params& p, int kv, int device, size_t ws_bytes, cudaStream_t stream) {
  const int hp = hp_for(p.kv_heads, p.qc, kv, p.q_al16, p.G);
  const bool cp = hp == 2 && p.qc > 1;  // chunk pairs
  const int S = num_work_ctas(device, kv, hp, p.head_dim, cp);
  if (S <= 0) return fail(FK_ERR_CUDA, "could not size the persistent grid on device %d", device);
  p.num_ctas = S;
  const int kvq = p.kv_heads * p.qc;  // (KV head, query chunk) pairs per sequence
  const WsLayout wl(ws_bytes, p.B, kvq, ws_ctas(S, hp));
  if (!wl.fits(ws_bytes, p.B, kvq))
    return fail(FK_ERR_WORKSPACE, "workspace too small: %zu bytes < %zu required", ws_bytes,
                WsLayout::min_bytes(p.B, kvq, ws_ctas(S, hp)));
  p.ws_cnt = static_cast<long long>(wl.cnt);
  p.ws_ml = static_cast<long long>(wl.ml);
  p.ws_acc = static_cast<long long>(wl.acc);
  if (p.B == 0) return FK_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != device) cudaSetDevice(device);
  prof_mark(0, stream);
  // e4m3 KV with bf16 or e4m3 Q copied raw: the consumers convert it
  const bool qconv = kv == FK_DTYPE_E4M3 && p.q_al16 && p.q_dtype != FK_DTYPE_F16;
#define FK_L(KVT, H, DD, CC, QQ) launch_one<KVT, LAYOUT, H, DD, CC, QQ>(p, S, device, stream)
#define FK_L_D(KVT, DD, QQ) \
  (cp ? FK_L(KVT, 2, DD, true, QQ) : hp == 2 ? FK_L(KVT, 2, DD, false, QQ) : FK_L(KVT, 1, DD, false, QQ))
  int rc;
  if (kv == FK_DTYPE_F16) rc = p.head_dim == 64 ? FK_L_D(FK_DTYPE_F16, 64, false) : FK_L_D(FK_DTYPE_F16, 128, false);
  else if (kv == FK_DTYPE_BF16) rc = p.head_dim == 64 ? FK_L_D(FK_DTYPE_BF16, 64, false) : FK_L_D(FK_DTYPE_BF16, 128, false);
  else if (hp == 4) rc = qconv ? FK_L(FK_DTYPE_E4M3, 4, 128, false, true) : FK_L(FK_DTYPE_E4M3, 4, 128, false, false);
  else rc = qconv ? FK_L_D(FK_DTYPE_E4M3, 128, true) : FK_L_D(FK_DTYPE_E4M3, 128, false);
#undef FK_L_D
#undef FK_L
  if (rc == FK_OK) {
    prof_mark(1, stream);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = fail(FK_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
  }
  if (prev != device) cudaSetDevice(prev);
  return rc;
}

// Q is read as element pairs (32-bit words for 16-bit Q, 16-bit for e4m3).
int check_q_align(const void* q, int q_dtype, int64_t sq_b, int64_t sq_h) {
  const uintptr_t a = (q_dtype == FK_DTYPE_E4M3) ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(q) % a) != 0 || (sq_b & 1) || (sq_h & 1))
    return fail(FK_ERR_INVALID_ARG, "q must be %d-byte aligned with even batch/head strides", static_cast<int>(a));
  return FK_OK;
}

void fill_common(Params& p, const void* q, int64_t sq_b, int64_t sq_h, void* out, int64_t so_b, int64_t so_h,
                 const float* s_aux, int batch, int q_heads, int kv_heads, int head_dim, int q_dtype, int out_dtype,
                 const float* scale_q, const float* scale_k, const float* scale_v, void* ws) {
  p.q = q;
  p.head_dim = head_dim;
  p.wait_ns = g_wait_ns.load();
  p.inject = g_inject.load();
  p.q_sb = sq_b;
  p.q_sh = sq_h;
  p.out = out;
  p.o_sb = so_b;
  p.o_sh = so_h;
  p.s_aux = s_aux;
  p.B = batch;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.G = q_heads / kv_heads;
  p.q_dtype = q_dtype;
  p.out_dtype = out_dtype;
  p.scale_q = scale_q;
  p.scale_k = scale_k;
  p.scale_v = scale_v;
  p.ws = static_cast<unsigned char*>(ws);
  p.qc = qc_for(q_heads, kv_heads);
  p.o_al8 = ((reinterpret_cast<uintptr_t>(out) & 7) == 0 && (so_b & 3) == 0 && (so_h & 3) == 0) ? 1 : 0;
  const int64_t qes = (q_dtype == FK_DTYPE_E4M3) ? 1 : 2;
  p.q_al16 = ((reinterpret_cast<uintptr_t>(q) & 15) == 0 && ((sq_b * qes) & 15) == 0 && ((sq_h * qes) & 15) == 0) ? 1 : 0;
}

}  // namespace fk

// ==========================================================================
// C ABI
// ==========================================================================
using namespace fk;

extern "C" int fk_version(void) { return 100; }

extern "C" const char* fk_last_error(void) { return g_err.c_str(); }

extern "C" size_t fk_decode_workspace_bytes_gqa(int device, int batch, int q_heads, int kv_heads, int kv_dtype) {
  if (batch < 0 || kv_heads <= 0 || q_heads <= 0 || q_heads % kv_heads != 0) {
    fail(FK_ERR_INVALID_ARG, "bad sizes");
    return 0;
  }
  const int qc = qc_for(q_heads, kv_heads);
  const int hp = hp_for(kv_heads, qc);
  int S = num_work_ctas_any_d(device, kv_dtype, hp, hp == 2 && qc > 1);
  if (S <= 0) {
    fail(FK_ERR_CUDA, "could not size the persistent grid on device %d", device);
    return 0;
  }
  // an e4m3 call may run four-head items (it depends on Q's alignment)
  const int hp4 = hp_for(kv_heads, qc, kv_dtype, 1, q_heads / kv_heads);
  if (hp4 == 4) {
    const int S4 = num_work_ctas(device, kv_dtype, 4);
    if (S4 <= 0) {
      fail(FK_ERR_CUDA, "could not size the persistent grid on device %d", device);
      return 0;
    }
    S = S > ws_ctas(S4, 4) ? S : ws_ctas(S4, 4);
  }
  return WsLayout::min_bytes(batch, kv_heads * qc, S);
}

extern "C" size_t fk_decode_workspace_bytes(int device, int batch, int kv_heads, int kv_dtype) {
  return fk_decode_workspace_bytes_gqa(device, batch, kv_heads, kv_heads, kv_dtype);
}

namespace fk {

// Argument checks and tensor maps of a varlen call, everything short of the
// launch (shared by the workspace and the allocation-free entry points, so
// that the latter touches its scratch only for a call that will launch).
// Returns FK_EMPTY for an empty batch.
int varlen_prepare(Params& p, int* device, const void* q, const void* k_varlen, const void* v_varlen,
                   const int32_t* cu_seqlens_k, const float* s_aux, void* out, int batch, int q_heads, int kv_heads,
                   int head_dim, int64_t total_tokens, int dtype, int64_t sq_b, int64_t sq_h, int64_t sk_t,
                   int64_t sk_h, int64_t sv_t, int64_t sv_h, int64_t so_b, int64_t so_h, void* workspace) {
  int rc = common_checks(q, k_varlen, v_varlen, out, batch, q_heads, kv_heads, head_dim, dtype, dtype, dtype,
                         workspace, device);
  if (rc != FK_OK) return rc;
  if ((rc = check_q_align(q, dtype, sq_b, sq_h)) != FK_OK) return rc;
  if (!is16(dtype)) return fail(FK_ERR_UNSUPPORTED, "varlen decode takes f16 or bf16 tensors");
  if (cu_seqlens_k == nullptr) return fail(FK_ERR_INVALID_ARG, "cu_seqlens_k must be non-null");
  if (total_tokens < 0 || total_tokens > 0x7fffffffLL) return fail(FK_ERR_INVALID_ARG, "bad total_tokens");
  if (((sk_t | sk_h | sv_t | sv_h) * 2) % 16 != 0)
    return fail(FK_ERR_INVALID_ARG, "k/v strides must be multiples of 16 bytes");
  memset(&p, 0, sizeof(p));
  fill_common(p, q, sq_b, sq_h, out, so_b, so_h, s_aux, batch, q_heads, kv_heads, head_dim, dtype, dtype, nullptr, nullptr,
              nullptr, workspace);
  p.lens = cu_seqlens_k;
  const uint64_t T = static_cast<uint64_t>(total_tokens > 0 ? total_tokens : 1);
  const uint32_t hp = static_cast<uint32_t>(hp_for(kv_heads, qc_for(q_heads, kv_heads), dtype, p.q_al16, q_heads / kv_heads));
  const uint32_t hb = box_heads(static_cast<int>(hp), qc_for(q_heads, kv_heads));
  // 16-bit rows as (64 dims, T rows, D/64 halves [128 B apart], heads): one
  // box {64, 64/hp, D/64, hp} per stage lands as [head][half][rows][64].
  const uint32_t nh = static_cast<uint32_t>(head_dim / 64);
  const uint64_t dims[4] = {64, T, nh, static_cast<uint64_t>(kv_heads)};
  const uint32_t box[4] = {64, tile_rows(dtype, head_dim) / hp, nh, hb};
  const uint64_t ks[3] = {static_cast<uint64_t>(sk_t) * 2, 128, static_cast<uint64_t>(sk_h) * 2};
  const uint64_t vs[3] = {static_cast<uint64_t>(sv_t) * 2, 128, static_cast<uint64_t>(sv_h) * 2};
  if ((rc = encode_map(&p.tk, dtype, 4, k_varlen, dims, ks, box)) != FK_OK) return rc;
  return encode_map(&p.tv, dtype, 4, v_varlen, dims, vs, box);
}

}  // namespace fk

extern "C" int fk_flash_decode_gqa_varlen(const void* q, const void* k_varlen, const void* v_varlen,
                                          const int32_t* cu_seqlens_k, const float* s_aux, void* out, int batch,
                                          int q_heads, int kv_heads, int head_dim, int64_t total_tokens, int dtype,
                                          int64_t sq_b, int64_t sq_h, int64_t sk_t, int64_t sk_h, int64_t sv_t,
                                          int64_t sv_h, int64_t so_b, int64_t so_h, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  int device = 0;
  Params p;
  const int rc = varlen_prepare(p, &device, q, k_varlen, v_varlen, cu_seqlens_k, s_aux, out, batch, q_heads, kv_heads,
                                head_dim, total_tokens, dtype, sq_b, sq_h, sk_t, sk_h, sv_t, sv_h, so_b, so_h,
                                workspace);
  if (rc == FK_EMPTY) return FK_OK;
  if (rc != FK_OK) return rc;
  return launch<VARLEN>(p, dtype, device, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int fk_flash_decode_gqa_hf_dense(const void* q, const void* k_cache, const void* v_cache,
                                            const int32_t* cache_lens, const int32_t* start_k_offsets,
                                            const float* s_aux, void* out, int batch, int q_heads, int kv_heads,
                                            int head_dim, int64_t max_seqlen, int q_dtype, int kv_dtype,
                                            int out_dtype, const float* scale_q, const float* scale_k,
                                            const float* scale_v, int64_t sq_b, int64_t sq_h, int64_t sk_b,
                                            int64_t sk_h, int64_t sk_s, int64_t sv_b, int64_t sv_h, int64_t sv_s,
                                            int64_t so_b, int64_t so_h, void* workspace, size_t workspace_bytes,
                                            void* stream) {
  int device = 0;
  int rc = common_checks(q, k_cache, v_cache, out, batch, q_heads, kv_heads, head_dim, q_dtype, kv_dtype, out_dtype,
                         workspace, &device);
  if (rc == FK_EMPTY) return FK_OK;
  if (rc != FK_OK) return rc;
  if ((rc = check_q_align(q, q_dtype, sq_b, sq_h)) != FK_OK) return rc;
  if (cache_lens == nullptr) return fail(FK_ERR_INVALID_ARG, "cache_lens must be non-null");
  if (max_seqlen <= 0 || max_seqlen > 0x7fffffffLL) return fail(FK_ERR_INVALID_ARG, "bad max_seqlen");
  const int es = (kv_dtype == FK_DTYPE_E4M3) ? 1 : 2;
  if (((sk_b | sk_h | sk_s | sv_b | sv_h | sv_s) * es) % 16 != 0)
    return fail(FK_ERR_INVALID_ARG, "k/v cache strides must be multiples of 16 bytes");
  Params p;
  memset(&p, 0, sizeof(p));
  fill_common(p, q, sq_b, sq_h, out, so_b, so_h, s_aux, batch, q_heads, kv_heads, head_dim, q_dtype, out_dtype, scale_q,
              scale_k, scale_v, workspace);
  p.lens = cache_lens;
  p.starts = start_k_offsets;
  p.max_tokens = max_seqlen;
  const uint32_t hp = static_cast<uint32_t>(hp_for(kv_heads, qc_for(q_heads, kv_heads), kv_dtype, p.q_al16, q_heads / kv_heads));
  const uint32_t hb = box_heads(static_cast<int>(hp), qc_for(q_heads, kv_heads));
  const uint64_t Bd = static_cast<uint64_t>(batch > 0 ? batch : 1);
  if (kv_dtype == FK_DTYPE_E4M3) {
    // (128 dims, S rows, heads, batch): box {128, 64/hp, hp, 1} -> [head][rows][128]
    const uint64_t dims[4] = {HEAD_DIM, static_cast<uint64_t>(max_seqlen), static_cast<uint64_t>(kv_heads), Bd};
    const uint32_t box[4] = {128, tile_rows(kv_dtype, head_dim) / hp, hb, 1};
    const uint64_t ks[3] = {static_cast<uint64_t>(sk_s), static_cast<uint64_t>(sk_h), static_cast<uint64_t>(sk_b)};
    const uint64_t vs[3] = {static_cast<uint64_t>(sv_s), static_cast<uint64_t>(sv_h), static_cast<uint64_t>(sv_b)};
    if ((rc = encode_map(&p.tk, kv_dtype, 4, k_cache, dims, ks, box)) != FK_OK) return rc;
    if ((rc = encode_map(&p.tv, kv_dtype, 4, v_cache, dims, vs, box)) != FK_OK) return rc;
  } else {
    // (64 dims, S rows, D/64 halves, heads, batch): box {64, 64/hp, D/64, hp, 1}
    // -> [head][half][rows][64]
    const uint32_t nh = static_cast<uint32_t>(head_dim / 64);
    const uint64_t dims[5] = {64, static_cast<uint64_t>(max_seqlen), nh, static_cast<uint64_t>(kv_heads), Bd};
    const uint32_t box[5] = {64, tile_rows(kv_dtype, head_dim) / hp, nh, hb, 1};
    const uint64_t ks[4] = {static_cast<uint64_t>(sk_s) * 2, 128, static_cast<uint64_t>(sk_h) * 2,
                            static_cast<uint64_t>(sk_b) * 2};
    const uint64_t vs[4] = {static_cast<uint64_t>(sv_s) * 2, 128, static_cast<uint64_t>(sv_h) * 2,
                            static_cast<uint64_t>(sv_b) * 2};
    if ((rc = encode_map(&p.tk, kv_dtype, 5, k_cache, dims, ks, box)) != FK_OK) return rc;
    if ((rc = encode_map(&p.tv, kv_dtype, 5, v_cache, dims, vs, box)) != FK_OK) return rc;
  }
  return launch<DENSE>(p, kv_dtype, device, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int fk_paged_flash_decode(const void* q, const void* k_pool, const void* v_pool,
                                     const int32_t* block_table, const int32_t* seq_lens, const float* s_aux,
                                     void* out, int batch, int q_heads, int kv_heads, int head_dim,
                                     int64_t num_pages, int page_size, int max_blocks, int q_dtype, int kv_dtype,
                                     int out_dtype, const float* scale_q, const float* scale_k,
                                     const float* scale_v, int64_t sq_b, int64_t sq_h, int64_t sk_p, int64_t sk_h,
                                     int64_t sk_s, int64_t sv_p, int64_t sv_h, int64_t sv_s, int64_t bt_b,
                                     int64_t so_b, int64_t so_h, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  int device = 0;
  int rc = common_checks(q, k_pool, v_pool, out, batch, q_heads, kv_heads, head_dim, q_dtype, kv_dtype, out_dtype,
                         workspace, &device);
  if (rc == FK_EMPTY) return FK_OK;
  if (rc != FK_OK) return rc;
  if ((rc = check_q_align(q, q_dtype, sq_b, sq_h)) != FK_OK) return rc;
  if (page_size != PAGE) return fail(FK_ERR_UNSUPPORTED, "page_size must be 16 (got %d)", page_size);
  if (block_table == nullptr || seq_lens == nullptr)
    return fail(FK_ERR_INVALID_ARG, "block_table and seq_lens must be non-null");
  if (num_pages <= 0 || num_pages > 0x7fffffffLL) return fail(FK_ERR_INVALID_ARG, "bad num_pages");
  if (max_blocks < 0) return fail(FK_ERR_INVALID_ARG, "bad max_blocks");
  const int es = (kv_dtype == FK_DTYPE_E4M3) ? 1 : 2;
  if (((sk_p | sk_h | sk_s | sv_p | sv_h | sv_s) * es) % 16 != 0)
    return fail(FK_ERR_INVALID_ARG, "k/v pool strides must be multiples of 16 bytes");
  if (num_pages > 0x7fffffffLL) return fail(FK_ERR_INVALID_ARG, "num_pages too large");
  Params p;
  memset(&p, 0, sizeof(p));
  fill_common(p, q, sq_b, sq_h, out, so_b, so_h, s_aux, batch, q_heads, kv_heads, head_dim, q_dtype, out_dtype, scale_q,
              scale_k, scale_v, workspace);
  p.lens = seq_lens;
  p.bt = block_table;
  p.bt_sb = bt_b;
  p.max_blocks = max_blocks;
  p.num_pages = static_cast<int>(num_pages);
  const uint32_t hp = static_cast<uint32_t>(hp_for(kv_heads, qc_for(q_heads, kv_heads), kv_dtype, p.q_al16, q_heads / kv_heads));
  const uint32_t hb = box_heads(static_cast<int>(hp), qc_for(q_heads, kv_heads));
  if (kv_dtype == FK_DTYPE_E4M3) {
    // [P, KVH, 16, 128] bytes: one box {128, 16, hp, 1} per page -> [head][16][128]
    const uint64_t dims[4] = {HEAD_DIM, PAGE, static_cast<uint64_t>(kv_heads), static_cast<uint64_t>(num_pages)};
    const uint32_t box[4] = {128, PAGE, hb, 1};
    const uint64_t ks[3] = {static_cast<uint64_t>(sk_s), static_cast<uint64_t>(sk_h), static_cast<uint64_t>(sk_p)};
    const uint64_t vs[3] = {static_cast<uint64_t>(sv_s), static_cast<uint64_t>(sv_h), static_cast<uint64_t>(sv_p)};
    if ((rc = encode_map(&p.tk, kv_dtype, 4, k_pool, dims, ks, box)) != FK_OK) return rc;
    if ((rc = encode_map(&p.tv, kv_dtype, 4, v_pool, dims, vs, box)) != FK_OK) return rc;
  } else {
    // 16-bit: the head dim is split into (64 dims, D/64 halves); the half index
    // is the third dimension (stride 128 B), so one box {64, 16, D/64, hp}
    // carries a page for the item's heads and lands as [head][half][16][64].
    const uint32_t nh = static_cast<uint32_t>(head_dim / 64);
    const uint64_t dims[5] = {64, PAGE, nh, static_cast<uint64_t>(kv_heads), static_cast<uint64_t>(num_pages)};
    const uint32_t box[5] = {64, PAGE, nh, hb, 1};
    const uint64_t ks[4] = {static_cast<uint64_t>(sk_s) * 2, 128, static_cast<uint64_t>(sk_h) * 2,
                            static_cast<uint64_t>(sk_p) * 2};
    const uint64_t vs[4] = {static_cast<uint64_t>(sv_s) * 2, 128, static_cast<uint64_t>(sv_h) * 2,
                            static_cast<uint64_t>(sv_p) * 2};
    if ((rc = encode_map(&p.tk, kv_dtype, 5, k_pool, dims, ks, box)) != FK_OK) return rc;
    if ((rc = encode_map(&p.tv, kv_dtype, 5, v_pool, dims, vs, box)) != FK_OK) return rc;
  }
  return launch<PAGED>(p, kv_dtype, device, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int fk_profile_begin(int max_launches) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  if (max_launches <= 0) return fail(FK_ERR_INVALID_ARG, "max_launches must be positive");
  if (g_prof.ev != nullptr) {
    for (int i = 0; i < 2 * g_prof.cap; ++i) cudaEventDestroy(g_prof.ev[i]);
    delete[] g_prof.ev;
  }
  g_prof.ev = new cudaEvent_t[2 * max_launches];
  for (int i = 0; i < 2 * max_launches; ++i) {
    const cudaError_t e = cudaEventCreate(&g_prof.ev[i]);
    if (e != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaEventDestroy(g_prof.ev[j]);
      delete[] g_prof.ev;
      g_prof.ev = nullptr;
      g_prof.cap = 0;
      g_prof.on = false;
      return fail(FK_ERR_CUDA, "cudaEventCreate: %s", cudaGetErrorString(e));
    }
  }
  g_prof.cap = max_launches;
  g_prof.n = 0;
  g_prof.on = true;
  return FK_OK;
}

extern "C" int fk_profile_end(float* kernel_ms, int* launches) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  g_prof.on = false;
  float total = 0.f;
  for (int i = 0; i < g_prof.n; ++i) {
    float a = 0.f;
    if (cudaEventSynchronize(g_prof.ev[2 * i + 1]) != cudaSuccess) return fail(FK_ERR_CUDA, "event sync failed");
    cudaEventElapsedTime(&a, g_prof.ev[2 * i], g_prof.ev[2 * i + 1]);
    total += a;
  }
  if (kernel_ms) *kernel_ms = total;
  if (launches) *launches = g_prof.n;
  return FK_OK;
}

extern "C" int fk_debug_configure(unsigned long long wait_ns, int inject) {
  if (wait_ns < 1000000ull || wait_ns > 60000000000ull)
    return fail(FK_ERR_INVALID_ARG, "wait_ns must be in [1 ms, 60 s]");
  if (inject != 0 && inject != 1) return fail(FK_ERR_INVALID_ARG, "inject must be 0 or 1");
  g_wait_ns.store(wait_ns);
  g_inject.store(inject);
  return FK_OK;
}

extern "C" int fk_decode_num_ctas(int device, int kv_dtype, int kv_heads) {
  return num_work_ctas(device, kv_dtype, hp_for(kv_heads));
}

// ==========================================================================
// Allocation-free variant of the varlen decode.
//
// For callers that must not allocate device memory at all -- for example a
// plugin that runs inside a host framework owning every allocation, or code
// running where cudaMalloc is forbidden after start-up -- the scratch
// (status word, arrival counters, segment partials) lives in the file-scope
// array below instead of a caller-provided workspace.  Every GPU that loads
// this library holds the array until the process exits.
// ==========================================================================
namespace fk {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(8) << 20;  // 8 MiB: up to ~1000 segments
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch, resolved once per device.  In host code
// the array's name is only a host-side stand-in, never a device pointer.
int noalloc_scratch(int device, void** out) {
  static void* addr[64] = {};
  static std::mutex mu;
  if (device < 0 || device >= 64) return fail(FK_ERR_INVALID_ARG, "device index %d out of range", device);
  std::lock_guard<std::mutex> lk(mu);
  if (addr[device] == nullptr) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess || p == nullptr)
      return fail(FK_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
    addr[device] = p;
  }
  *out = addr[device];
  return FK_OK;
}

}  // namespace fk

extern "C" size_t fk_noalloc_scratch_bytes(void) { return NOALLOC_SCRATCH_BYTES; }

extern "C" int fk_flash_decode_gqa_varlen_noalloc(const void* q, const void* k_varlen, const void* v_varlen,
                                                  const int32_t* cu_seqlens_k, const float* s_aux, void* out,
                                                  int batch, int q_heads, int kv_heads, int head_dim,
                                                  int64_t total_tokens, int dtype, int64_t sq_b, int64_t sq_h,
                                                  int64_t sk_t, int64_t sk_h, int64_t sv_t, int64_t sv_h,
                                                  int64_t so_b, int64_t so_h, void* stream) {
  // Every argument is checked (and the tensor maps built) before the scratch
  // is touched: a refused call queues nothing on the stream.  The workspace
  // argument of the checks only has to be non-null here.
  int device = 0;
  Params p;
  int rc = varlen_prepare(p, &device, q, k_varlen, v_varlen, cu_seqlens_k, s_aux, out, batch, q_heads, kv_heads,
                          head_dim, total_tokens, dtype, sq_b, sq_h, sk_t, sk_h, sv_t, sv_h, so_b, so_h,
                          reinterpret_cast<void*>(uintptr_t(1)));
  if (rc == FK_EMPTY) return FK_OK;
  if (rc != FK_OK) return rc;
  const int qc = qc_for(q_heads, kv_heads);
  const int hp = hp_for(kv_heads, qc);
  const int S = num_work_ctas(device, dtype, hp, head_dim, hp == 2 && qc > 1);
  if (S <= 0) return fail(FK_ERR_CUDA, "could not size the persistent grid on device %d", device);
  const long long items = static_cast<long long>(batch) * kv_heads * qc;
  const WsLayout wl(NOALLOC_SCRATCH_BYTES, batch, kv_heads * qc, S);
  if (!wl.fits(NOALLOC_SCRATCH_BYTES, batch, kv_heads * qc))
    return fail(FK_ERR_WORKSPACE,
                "batch*kv_heads*ceil(G/8) = %lld needs %zu bytes of scratch; the allocation-free entry point has a "
                "fixed %zu-byte scratch, which holds batch*kv_heads*ceil(G/8) + %d (resident CTAs) <= %zu",
                items, WsLayout::min_bytes(batch, kv_heads * qc, S), NOALLOC_SCRATCH_BYTES, S,
                (NOALLOC_SCRATCH_BYTES - 256 - 1024) / SEG_BYTES);
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(device, &scratch)) != FK_OK) return rc;
  p.ws = static_cast<unsigned char*>(scratch);
  // The arrival counters must start at zero: clear them on the caller's
  // stream (a memset, not an allocation).  The status word before them is
  // left alone: it collects FK_STATUS_* bits until fk_noalloc_read_status
  // clears it.
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != device) cudaSetDevice(device);
  const cudaError_t e = cudaMemsetAsync(static_cast<unsigned char*>(scratch) + wl.cnt, 0, wl.ml - wl.cnt,
                                        static_cast<cudaStream_t>(stream));
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(FK_ERR_CUDA, "clearing the scratch failed: %s", cudaGetErrorString(e));
  return launch<VARLEN>(p, dtype, device, NOALLOC_SCRATCH_BYTES, static_cast<cudaStream_t>(stream));
}

extern "C" int fk_noalloc_read_status(int device, int* status, int clear) {
  if (status == nullptr) return fail(FK_ERR_INVALID_ARG, "status must be non-null");
  void* scratch = nullptr;
  int rc = noalloc_scratch(device, &scratch);
  if (rc != FK_OK) return rc;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != device) cudaSetDevice(device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(status, scratch, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear && *status != 0) e = cudaMemset(scratch, 0, sizeof(int));
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(FK_ERR_CUDA, "reading the scratch status failed: %s", cudaGetErrorString(e));
  return FK_OK;
}

#ifdef FK_TRACE
extern "C" int fk_trace_read(unsigned long long* host, int n) {
  return cudaMemcpyFromSymbol(host, g_trace, sizeof(unsigned long long) * 32 * n) == cudaSuccess ? 0 : 1;
}
#endif
