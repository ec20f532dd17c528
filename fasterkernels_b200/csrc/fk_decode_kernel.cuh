// fk_decode_kernel.cuh -- the device side of fk_decode.cu: constants, shared-
// memory layouts, work-item mapping and the persistent decode kernel.
//
// Work decomposition ("stream-K" over KV granules).  A work item is one
// sequence b x HP KV heads (HP = 2 when kv_heads is even), or, for groups of
// more than 8 query heads, one KV head x two chunks of at most 8 query heads.
// Each item owns ceil(len_b / 16) granules of 16 tokens; items are laid end
// to end (b-major) into one stream of U granules, and CTA c of the
// persistent grid (S CTAs, S = resident CTAs on the device) takes granules
// [c*per, (c+1)*per) with per = max(ceil(U/S), 4).  Every CTA therefore
// streams the same number of KV bytes whatever the length distribution, and
// the plan is derived on the device from the lengths alone (no host sync,
// CUDA-graph safe).  The piece of item i inside CTA c is a segment with id
// c + i (unique, < S + items).  A CTA that holds a whole item normalises and
// writes the output itself; otherwise it stores the segment's (max, sum,
// acc) partial in the workspace and bumps the item's arrival counter; the CTA
// that brings the counter to the item's segment count merges the partials in
// CTA order with the sink term (log-sum-exp combine) and re-arms the counter.
// One launch per decode call; no CTA ever waits for another.
//
// Split pass, per CTA: one producer warp walks the plan, copies each
// segment's Q rows with cp.async and issues TMA tile loads (64 rows, or 128
// at head dim 64, of K and of V per stage, 128-byte swizzled) into an
// mbarrier ring; four consumer warps each take blocks of 16 rows of every
// tile and run QK^T and PV on the tensor cores with mma.sync m16n8k16,
// tokens as the M dimension and up to 8 query heads as N, keeping a private
// online-softmax state; two epilogue warps merge the four warps' states of
// each finished segment and write outputs or partials.  FP8 e4m3 K/V are
// widened to f16 in registers; scale_k folds into the logit scale and
// scale_v into the final output.
//
// Layouts (address policies of the producer; D = head dim, 128 or 64):
//   VARLEN  k[T, KVH, D]          tensor map coords (d, t, half, h)
//   DENSE   k[B, KVH, S, D]       tensor map coords (d, s, half, h, b)
//   PAGED   pool[P, KVH, 16, D]   tensor map coords (d, slot, half, h, page)
// (e4m3 rows are a single 128-byte half, so their maps drop that coordinate.)
// The plan, the tile sequence and the arithmetic do not depend on the
// layout, so paged and contiguous results are bit-identical.
#pragma once
#include <cuda.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/fk_decode.h"
#include "fk_ptx.cuh"

namespace fk {

constexpr int HEAD_DIM = 128;  // largest head dim; workspace records, epilogue slots and Q rows are sized for it
constexpr int GPAD = 8;        // MMA N: query heads of one KV group, padded
constexpr int CWARPS = 4;      // consumer warps, 16 tokens of each tile apiece
constexpr int EWARPS = 2;      // epilogue warps: segment merge / output / partials
constexpr int THREADS = (CWARPS + 1 + EWARPS) * 32;
constexpr int ETHREADS = EWARPS * 32;
constexpr int HPMAX = 2;       // KV heads per work item of the 16-bit kernels (2 when kv_heads is even)
constexpr int GMAX = HPMAX * 8; // query-head slots per workspace record
// e4m3 KV with kv_heads % 4 == 0 and groups of at most 8 query heads runs four
// KV heads per item (one 8 KB TMA box per page instead of two 4 KB boxes);
// its segment record spans two consecutive 16-slot records.
constexpr int PAGE = 16;       // tokens per granule (= page size)
constexpr int MIN_PER = 4;     // minimum granules per CTA (one tile)
constexpr int FK_EMPTY = -1;   // internal: common_checks found an empty batch
constexpr float LOG2E = 1.4426950408889634f;
// log2 headroom before the running max is moved (see the consumers); bf16 P
// keeps the exact running max (0): its 8-bit mantissa leaves no slack in the
// reference's 1e-3 tolerance.
constexpr float LAZY_MAX_F16 = 8.f;
constexpr float NEG_INF = -__builtin_huge_valf();

enum Layout { VARLEN = 0, DENSE = 1, PAGED = 2 };
enum Flags { F_FIRST = 1, F_LAST = 2, F_WHOLE = 4, F_END = 8 };

// Per KV element type and head dim D (128; 64 for 16-bit KV).
// Per KV element type, head dim D and chunk-pair mode CP (groups of more
// than 8 query heads: the item's two head slots are two query chunks of one
// KV head, so a stage holds that one head's tile).
template <int KV, int D, bool CP = false>
struct KvCfg {
  static constexpr bool FP8 = (KV == FK_DTYPE_E4M3);
  static constexpr bool BF16 = (KV == FK_DTYPE_BF16);
  static_assert(D == 128 || (D == 64 && !FP8), "head dim 128, or 64 with 16-bit KV");
  static constexpr int ES = FP8 ? 1 : 2;                     // bytes per element
  static constexpr int NH = D * ES / 128;                    // 128-byte halves per row
  static constexpr int KD = D / 16;                          // MMA k-steps (QK) / dim tiles (PV)
  // Rows (tokens x item heads) per stage: D = 64 doubles them so that a stage
  // carries as many bytes as at D = 128; each consumer warp then takes
  // TILE / 64 blocks of 16 rows.
  static constexpr int TILE = (D == 64) ? 128 : 64;
  static constexpr int HPL = CP ? 1 : 2;                     // KV heads laid out per stage (at most)
  static constexpr int TILE_BYTES = TILE / 2 * HPL * D * ES; // K (or V) bytes per stage
  static constexpr int PAGE_BYTES = PAGE * D * ES;           // one page of one head's K (or V)
  // Chunk pairs do twice the MMA and softmax work per byte: their smaller
  // stages let two CTAs share an SM (16-bit) or keep more stages (e4m3).
  static constexpr int STAGES = FP8 ? (CP ? 6 : 4) : (CP ? 4 : 5);
  static constexpr int NSLOT = (FP8 || CP) ? 1 : 2;          // epilogue slots (shared-memory budget)
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int MINB = (FP8 || CP) ? 2 : 1;           // resident CTAs per SM (at least)
  // Q slots: each segment's Q rows are staged in one of two slots, released
  // by the consumers once they hold them in registers.
  static constexpr int QSLOTS = 2;
};

// One epilogue slot: the four consumer warps' online-softmax states of a
// finished segment, handed to the epilogue warps.
struct EpiSlot {
  float cm[CWARPS][GPAD];
  float cl[CWARPS][GPAD];
  float cacc[CWARPS][GPAD][HEAD_DIM];
};

// Shared-memory tile layouts of one K (or V) stage: TT = TILE/HP tokens of each
// of the item's HP KV heads (one head's with chunk pairs), 128-byte swizzled
// (16-byte chunk index XOR row & 7).  A row of D elements is NH = D * ES /
// 128 halves of 128 bytes
// (16-bit D = 128: two 64-dim halves; 16-bit D = 64 and e4m3 D = 128: one).
//   VARLEN / DENSE: [head][half][TT rows][128 B]   one TMA box per stage
//   PAGED:          [page][head][half][16][128 B]  one TMA box per page
// Row r of head hh, 16-byte chunk c is at row_off(hh, r) + (c >> 3) *
// HALF_STRIDE + (((c & 7) ^ (r & 7)) << 4).  All bases are multiples of 1024
// bytes, so the swizzle line of row r is r & 7 everywhere.
template <int KV, int LAYOUT, int HP, int D, bool CP = false>
struct TileLayout {
  static constexpr bool PG = LAYOUT == 2;  // PAGED
  static constexpr int NH = KvCfg<KV, D, CP>::NH;
  static constexpr int TT = KvCfg<KV, D, CP>::TILE / HP;
  static constexpr int HS = CP ? 1 : HP;   // KV heads stored per stage
  static constexpr uint32_t HALF_STRIDE = PG ? 2048u : uint32_t(TT * 128);
  __device__ static __forceinline__ uint32_t row_off(int hh, int r) {
    if constexpr (PG) return uint32_t((r >> 4) * (HS * NH * 2048) + hh * (NH * 2048) + (r & 15) * 128);
    else return uint32_t(hh * (NH * TT * 128) + r * 128);
  }
};

struct Meta {
  int b, h, tok, valid, flags, seg, bad, c0, nseg, qslot, pad[2];
};

// Workspace layout (bytes), a function of the workspace SIZE W so that every
// launch on one buffer agrees on where the arrival counters live:
//   [0, 256)                 header (status word)
//   [256, 256 + 4*cap)       cnt[cap]: per-item arrival counters, cap =
//                            (W - 256) / SEG_BYTES; zero between launches
//   ml  (aligned 256)        float2[(S+I)*16]  segment (max, sum) per query-head slot
//   acc (aligned 256)        float[(S+I)*16*128] segment accumulators
// A launch with I = B*KVH items fits when I <= cap and acc + its size <= W.
// Partials of one launch can therefore never overwrite the counters another
// launch (of any shape) uses on the same buffer.
struct WsHeader {
  int status;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr size_t SEG_BYTES = 4 + GMAX * sizeof(float2) + GMAX * HEAD_DIM * sizeof(float);  // per segment (+1 counter)

struct WsLayout {
  size_t cap, cnt, ml, acc, need;
  WsLayout(size_t W, int B, int kvh, int S) {
    const size_t segs = static_cast<size_t>(S) + static_cast<size_t>(B) * kvh;
    cap = W > 256 ? (W - 256) / SEG_BYTES : 0;
    cnt = 256;
    ml = align_up(cnt + 4 * cap, 256);
    acc = align_up(ml + segs * GMAX * sizeof(float2), 256);
    need = acc + segs * GMAX * HEAD_DIM * sizeof(float);
  }
  bool fits(size_t W, int B, int kvh) const { return static_cast<size_t>(B) * kvh <= cap && need <= W; }
  // Smallest buffer size whose own layout fits (B, kvh, S).
  static size_t min_bytes(int B, int kvh, int S) {
    const size_t segs = static_cast<size_t>(S) + static_cast<size_t>(B) * kvh;
    return align_up(256 + segs * SEG_BYTES + 1024, 256);
  }
};

struct Params {
  CUtensorMap tk;  // K tensor map (64-byte aligned, first member)
  CUtensorMap tv;  // V tensor map
  const void* q;
  long long q_sb, q_sh;
  void* out;
  long long o_sb, o_sh;
  const int* lens;    // VARLEN: cu_seqlens[B+1]; DENSE: cache_lens[B]; PAGED: seq_lens[B]
  const int* starts;  // DENSE: start_k_offsets[B] or null
  const int* bt;      // PAGED: block table
  long long bt_sb;
  long long max_tokens;  // DENSE: cache rows per sequence
  long long ws_cnt, ws_ml, ws_acc;  // workspace region offsets (bytes)
  int max_blocks, num_pages;
  const float* s_aux;
  const float* scale_q;
  const float* scale_k;
  const float* scale_v;
  unsigned char* ws;
  int B, q_heads, kv_heads, G;
  int q_dtype, out_dtype;
  int num_ctas;
  int q_al16;  // q base and strides 16-byte aligned (rows can be copied with cp.async)
  int o_al8;   // out base and strides 8-byte aligned (four outputs per store)
  int qc;      // query chunks of at most 8 heads per KV head: ceil(G / 8)
  int head_dim;  // D (the kernel is instantiated per D; kept for host checks)
  unsigned long long wait_ns;  // bound of every mbarrier wait
  int inject;                  // test hook: 1 = each CTA's producer withholds its first stage
};

// Work items of a sequence and their two head slots hh < HP (an MMA N of 8
// query heads each).  A group of up to 8 query heads (qc = 1): item hi covers
// KV heads hi*HP .. + HP - 1, slot hh holds the group of KV head hi*HP + hh.
// Larger groups are cut into qc chunks of at most 8 query heads: with HP = 2
// the two slots of an item hold two chunks of ONE KV head, whose tile is
// loaded once and read by both slots' warps ("chunk pairs"); with HP = 1 each
// chunk is an item.  Slot hh holds query heads item_q(hi, hh, j) of KV head
// item_kv(hi), j < item_g(hi, hh) (0 for the empty second slot of an odd
// chunk count).
template <int HP>
__device__ __forceinline__ int item_kv(const Params& p, int hi) {
  if (p.qc == 1) return hi * HP;
  return HP == 2 ? hi / ((p.qc + 1) >> 1) : hi / p.qc;
}
template <int HP>
__device__ __forceinline__ int item_chunk(const Params& p, int hi, int hh) {
  if (p.qc == 1) return 0;
  return HP == 2 ? (hi % ((p.qc + 1) >> 1)) * 2 + hh : hi % p.qc;
}
template <int HP>
__device__ __forceinline__ int item_q(const Params& p, int hi, int hh, int j) {
  if (p.qc == 1) return (hi * HP + hh) * p.G + j;
  return item_kv<HP>(p, hi) * p.G + item_chunk<HP>(p, hi, hh) * 8 + j;
}
template <int HP>
__device__ __forceinline__ int item_g(const Params& p, int hi, int hh) {
  if (p.qc == 1) return p.G;
  return max(0, min(8, p.G - item_chunk<HP>(p, hi, hh) * 8));
}
// Items per sequence.
template <int HP>
__device__ __forceinline__ int items_per_seq(const Params& p) {
  if (p.qc == 1) return p.kv_heads / HP;
  return HP == 2 ? p.kv_heads * ((p.qc + 1) >> 1) : p.kv_heads * p.qc;
}

// Query row r (< item_rows) of item hi -> head slot hh and query head j
// within the slot.  Four-head items only exist for groups of at most 8
// query heads (one chunk).
template <int HP>
__device__ __forceinline__ int item_rows(const Params& p, int hi) {
  if constexpr (HP == 4) return 4 * p.G;
  else return item_g<HP>(p, hi, 0) + (HP == 2 ? item_g<HP>(p, hi, 1) : 0);
}
template <int HP>
__device__ __forceinline__ void item_row(const Params& p, int hi, int r, int& hh, int& j) {
  if constexpr (HP == 4) {
    hh = r / p.G;
    j = r - hh * p.G;
  } else {
    const int g0 = item_g<HP>(p, hi, 0);
    hh = r < g0 ? 0 : 1;
    j = r < g0 ? r : r - g0;
  }
}

// Effective length of sequence b and the coordinate of its first token.
template <int LAYOUT>
__device__ __forceinline__ int seq_len(const Params& p, int b, long long* tok0) {
  if constexpr (LAYOUT == VARLEN) {
    const int s = __ldg(p.lens + b), e = __ldg(p.lens + b + 1);
    *tok0 = s;
    return max(e - s, 0);
  } else if constexpr (LAYOUT == DENSE) {
    const int s = p.starts ? max(__ldg(p.starts + b), 0) : 0;
    const long long e = min(static_cast<long long>(__ldg(p.lens + b)), p.max_tokens);
    *tok0 = s;
    return static_cast<int>(max(e - s, 0ll));
  } else {
    *tok0 = 0;
    return max(__ldg(p.lens + b), 0);
  }
}

__device__ __forceinline__ long long warp_incl_scan(long long v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Two adjacent Q elements (even element index e) as raw bits: 32 bits for
// 16-bit Q, 16 bits for e4m3 Q.  Strides and the base are validated on the
// host to keep these loads aligned.
__device__ __forceinline__ uint32_t load_q_pair_raw(const Params& p, long long e) {
  if (p.q_dtype == FK_DTYPE_E4M3) return __ldg(reinterpret_cast<const unsigned short*>(static_cast<const unsigned char*>(p.q) + e));
  return __ldg(reinterpret_cast<const uint32_t*>(static_cast<const unsigned short*>(p.q) + e));
}

// Raw Q pair -> packed pair of the MMA element type.
template <bool MBF16>
__device__ __forceinline__ uint32_t q_pair_to_mma(const Params& p, uint32_t raw, float sq) {
  if (p.q_dtype == (MBF16 ? FK_DTYPE_BF16 : FK_DTYPE_F16)) return raw;
  float x0, x1;
  if (p.q_dtype == FK_DTYPE_E4M3) {
    x0 = __half2float(__half(__nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(raw & 0xff), __NV_E4M3))) * sq;
    x1 = __half2float(__half(__nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>((raw >> 8) & 0xff), __NV_E4M3))) * sq;
  } else if (p.q_dtype == FK_DTYPE_BF16) {
    x0 = __uint_as_float(raw << 16);
    x1 = __uint_as_float(raw & 0xffff0000u);
  } else {
    __half_raw a, b2;
    a.x = static_cast<unsigned short>(raw & 0xffff);
    b2.x = static_cast<unsigned short>(raw >> 16);
    x0 = __half2float(__half(a));
    x1 = __half2float(__half(b2));
  }
  return pack2<MBF16>(x0, x1);
}

__device__ __forceinline__ void store_out(const Params& p, long long idx, float v) {
  if (p.out_dtype == FK_DTYPE_BF16)
    static_cast<__nv_bfloat16*>(p.out)[idx] = __float2bfloat16_rn(v);
  else
    static_cast<__half*>(p.out)[idx] = __float2half_rn(v);
}

// Four consecutive outputs starting at element idx: one 8-byte store when the
// output allows it (p.o_al8: base and strides 8-byte aligned, idx a multiple
// of 4), else four.
__device__ __forceinline__ void store_out4(const Params& p, long long idx, float a, float b, float c, float d) {
  if (p.o_al8) {
    uint2 w;
    if (p.out_dtype == FK_DTYPE_BF16) {
      w.x = pack2<true>(a, b);
      w.y = pack2<true>(c, d);
    } else {
      w.x = pack2<false>(a, b);
      w.y = pack2<false>(c, d);
    }
    *reinterpret_cast<uint2*>(static_cast<unsigned short*>(p.out) + idx) = w;
  } else {
    store_out(p, idx, a);
    store_out(p, idx + 1, b);
    store_out(p, idx + 2, c);
    store_out(p, idx + 3, d);
  }
}

// Normalisation of query head qh with the oracle's sink formula.  L and the
// head's accumulators A are relative to its running max M (log2 domain):
// out = (A * e) / Lf * scale_v with e = 2^(M - Ms), Lf = L e + 2^(s - Ms),
// Ms = max(M, s); without a sink e = 1 and Lf = L.
__device__ __forceinline__ void sink_norm(float L, float M, const float* s_aux, int qh, float* e, float* Lf) {
  if (s_aux != nullptr) {
    const float s2 = __ldg(s_aux + qh) * LOG2E;
    const float Ms = fmaxf(M, s2);
    *e = exp2f(M - Ms);
    *Lf = L * *e + exp2f(s2 - Ms);
  } else {
    *e = 1.f;
    *Lf = L;
  }
}

__device__ __forceinline__ float norm_out(float A, float e, float Lf, float sv) {
  return Lf > 0.f ? ((A * e) / Lf) * sv : 0.f;
}

#ifdef FK_TRACE
// Per-CTA timeline for performance investigation builds (-DFK_TRACE):
// [start, first tile, consumer end (ns), segments, tiles, producer switch ns, producer acquire-wait ns,
//  consumer wait ns at first tiles of segments, consumer wait ns at other tiles, epilogue end (ns),
//  SM id, producer cycles in block-table lookup, in Q staging, in issue, per whole tile]
__device__ unsigned long long g_trace[4096][32];
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#endif

// ------------------------------------------------------------------------
// Split pass.
// ------------------------------------------------------------------------
// QC: the consumers convert Q staged raw (bf16 or e4m3 Q over e4m3 KV) to the
// MMA type as they load it; its own instantiation keeps that code out of the
// kernels that never need it.
template <int KV, int LAYOUT, int HP, int D, bool CP, bool QC>
__global__ void __launch_bounds__(THREADS, KvCfg<KV, D, CP>::MINB) decode_split_kernel(const __grid_constant__ Params p) {
  static_assert(!CP || HP == 2, "chunk pairs fill the two head slots of an item");
  static_assert(HP != 4 || (KV == FK_DTYPE_E4M3 && !CP), "four-head items are an e4m3 kernel");
  constexpr int GSR = (HP == 4) ? 4 * GPAD : GMAX;  // query-head slots per segment record
  static_assert(!QC || KV == FK_DTYPE_E4M3, "16-bit KV takes Q of its own type");
  using C = KvCfg<KV, D, CP>;
  using TL = TileLayout<KV, LAYOUT, HP, D, CP>;
  constexpr int KD = C::KD;
  constexpr int TT = C::TILE / HP;       // tokens per KV head in one stage
  constexpr int WPH = CWARPS / HP;       // consumer warps per KV head
  constexpr int PPT = TT / PAGE;         // pages per KV head in one stage
  constexpr int QWORDS = HP * GPAD * 64; // staged Q words per stage
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* stages = smem;
  static_assert(D <= HEAD_DIM, "head dim");
  EpiSlot* eslot = reinterpret_cast<EpiSlot*>(smem + C::STAGES * C::STAGE_BYTES);  // [NSLOT]
  Meta* emeta = reinterpret_cast<Meta*>(eslot + C::NSLOT);                         // [NSLOT]
  Meta* meta = emeta + C::NSLOT;                                                   // [STAGES]
  uint32_t* qstage = reinterpret_cast<uint32_t*>(meta + C::STAGES);                // [QSLOTS][QWORDS]
  uint64_t* full = reinterpret_cast<uint64_t*>(qstage + C::QSLOTS * QWORDS);       // [STAGES]
  uint64_t* empty = full + C::STAGES;                                              // [STAGES]
  uint64_t* efull = empty + C::STAGES;                                             // [NSLOT]
  uint64_t* eempty = efull + C::NSLOT;                                             // [NSLOT]
  uint64_t* qempty = eempty + C::NSLOT;                                            // [QSLOTS]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  WsHeader* hdr = reinterpret_cast<WsHeader*>(p.ws);
  int* cnt = reinterpret_cast<int*>(p.ws + p.ws_cnt);
  float2* ws_ml = reinterpret_cast<float2*>(p.ws + p.ws_ml);
  float* ws_acc = reinterpret_cast<float*>(p.ws + p.ws_acc);
  const int KVI = items_per_seq<HP>(p);
  __shared__ int s_last;
  __shared__ int s_eok[2][EWARPS];  // epilogue warps' wait outcomes, by iteration parity

#ifdef FK_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 4096) {
    for (int i = 1; i < 32; ++i) g_trace[blockIdx.x][i] = 0;
    g_trace[blockIdx.x][0] = gtimer();
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    g_trace[blockIdx.x][10] = smid;
  }
  unsigned long long tr_nseg = 0, tr_ntile = 0;
  bool tr_first = true;
#endif
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), CWARPS);
    }
    for (int s = 0; s < C::NSLOT; ++s) {
      mbar_init(smem_u32(&efull[s]), CWARPS * 32);
      mbar_init(smem_u32(&eempty[s]), ETHREADS);
    }
    for (int s = 0; s < C::QSLOTS; ++s) mbar_init(smem_u32(&qempty[s]), CWARPS);
    fence_mbar_init();
  }
  // Q rows 16-byte aligned: each segment's Q rows are copied raw into one of
  // the two Q slots by cp.async, completing on the stage's full barrier with
  // the KV tiles, and the consumers convert them to the MMA type (and apply
  // scale_q) as they load them; the padding rows (heads G..7) are zeroed
  // once, here.  Otherwise the producer converts Q through registers.
  const bool q_async = p.q_al16 != 0;
  // fewest query heads in a slot of any item
  const int gmin = p.qc == 1 ? p.G : (CP && (p.qc & 1)) ? 0 : (p.G % 8 == 0 ? 8 : p.G % 8);
  if (q_async && gmin < GPAD) {
    const int npad = GPAD - gmin;
    for (int u = threadIdx.x; u < C::QSLOTS * HP * npad * 16; u += THREADS) {
      const int row = u >> 4, c = u & 15;  // row over (Q slot, head, padding head)
      const int sh = row / npad, j = gmin + row % npad;
      reinterpret_cast<uint4*>(qstage + sh * (GPAD * 64) + j * 64)[c] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  // Programmatic dependent launch: this grid may start while the kernel
  // before it in the stream (a decode call, a KV append, a RoPE or projection
  // kernel) is still running.  Nothing above reads global memory; every input
  // (lengths, block table, Q, K/V, sinks, scales) is read after this wait,
  // which returns once the prerequisite grid has completed and its writes are
  // visible.
  grid_dependency_wait();
  // Plan, with every thread of the CTA: thread t sums the granules of
  // sequences [t*bpt, (t+1)*bpt) (independent loads, one round trip); each
  // warp scans its 32 sums in parallel, and every thread adds the totals of
  // the warps before its own to get its exclusive prefix.
  __shared__ long long s_psum[THREADS];
  __shared__ long long s_pexc[THREADS];
  __shared__ long long s_wtot[THREADS / 32];
  const int bpt = (p.B + THREADS - 1) / THREADS;
  {
    long long mysum = 0;
    const int b0 = threadIdx.x * bpt, b1 = min(b0 + bpt, p.B);
    for (int b = b0; b < b1; ++b) {
      long long t0;
      mysum += (seq_len<LAYOUT>(p, b, &t0) + PAGE - 1) / PAGE;
    }
    const long long inc = warp_incl_scan(mysum, lane);
    if (lane == 31) s_wtot[warp] = inc;
    __syncthreads();
    long long base = 0;
    for (int w = 0; w < warp; ++w) base += s_wtot[w];
    s_psum[threadIdx.x] = mysum;
    s_pexc[threadIdx.x] = base + inc - mysum;
  }
  __syncthreads();
#ifdef FK_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][16] = gtimer();
#endif
  // Let the next kernel in the stream start its CTAs as SMs free up (it
  // waits for this grid's completion before reading anything).
  grid_dependency_trigger();

  if (warp == CWARPS) {
    // ================================================================ producer
    if (lane == 0) {
      prefetch_tmap(&p.tk);
      prefetch_tmap(&p.tv);
    }
    const long long NI = KVI;
    const float psq = (p.scale_q != nullptr) ? __ldg(p.scale_q) : 1.f;

    const long long tot = s_pexc[THREADS - 1] + s_psum[THREADS - 1];  // granules of the whole batch
    const long long U = tot * NI;
    const long long S = p.num_ctas;
    const long long per = max((U + S - 1) / S, static_cast<long long>(MIN_PER));
    const long long start = static_cast<long long>(blockIdx.x) * per;
    const long long end = min(start + per, U);

    int stage = 0;
    uint32_t phase = 0;
    bool alive = true;
    // Test hook (off unless the host sets it): publish nothing for the first
    // stage, so the consumers' bounded wait on it runs out and the kernel
    // returns with FK_STATUS_TIMEOUT.  The later stages' copies are still
    // issued; on any timeout exit the producer waits (bounded) for every
    // stage it armed to land before the CTA leaves (see the end of this
    // branch).
    bool withhold = p.inject == 1;
    // Stages armed with copies (bit s) and the phase parity each was armed in.
    uint32_t armed = 0, armed_par = 0;
    // Claim the next ring slot (waits for the consumers to release it).
    auto acquire = [&]() -> bool {
      int ok = 1;
#ifdef FK_TRACE
      const unsigned long long tq0 = gtimer();
#endif
      if (lane == 0) ok = mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, p.wait_ns) ? 1 : 0;
#ifdef FK_TRACE
      if (lane == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][6] += gtimer() - tq0;
#endif
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok && lane == 0) atomicOr(&hdr->status, FK_STATUS_TIMEOUT);
      return ok != 0;
    };
    auto advance = [&]() {
      if (++stage == C::STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    };
    // Q slot of the next segment (waits for the consumers to release it).
    int qslot = 0;
    uint32_t qphase = 0;
    auto qacquire = [&]() -> bool {
      int ok = 1;
      if (lane == 0) ok = mbar_wait(smem_u32(&qempty[qslot]), qphase ^ 1u, p.wait_ns) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok && lane == 0) atomicOr(&hdr->status, FK_STATUS_TIMEOUT);
      return ok != 0;
    };

    // Q words of the next item, prefetched into registers: lane owns words
    // lane + 32k of the [HP][8 heads][64 pairs] block; paged: a window of 32
    // block-table entries (one per lane) + the next one.
    constexpr int QW = HP * GPAD * 64 / 32;
    uint32_t qpre[QW];
    int qpre_b = -1, qpre_h = -1;
    auto q_prefetch = [&](int bb, int ih) {
      const long long qb0 = static_cast<long long>(bb) * p.q_sb;
#pragma unroll
      for (int k = 0; k < QW; ++k) {
        const int idx = lane + 32 * k;
        const int hh = idx / (GPAD * 64), j = (idx >> 6) & (GPAD - 1), d = (idx & 63) * 2;
        const int qh = item_q<HP>(p, ih, hh, j);
        qpre[k] = (j < item_g<HP>(p, ih, hh) && d < D) ? load_q_pair_raw(p, qb0 + static_cast<long long>(qh) * p.q_sh + d)
                                                       : 0u;
      }
      qpre_b = bb;
      qpre_h = ih;
    };
#ifdef FK_TRACE
    long long tr_c[4] = {0, 0, 0, 0};  // producer cycles: block table, Q staging, issue, whole tile
#endif
    int win_b = -1;
    int win_p0 = 0;
    int bt_cur = -1, bt_nxt = -1;
    auto ld_bt = [&](int bb, int pg) -> int {
      return (pg < p.max_blocks) ? __ldg(p.bt + static_cast<long long>(bb) * p.bt_sb + pg) : -1;
    };

    if (start < end) {
      // Locate the first item of this CTA's granule range: the thread block
      // of sequences containing `start`, then the sequence inside it.
      int kt = -1;
      for (int base = 0; base < THREADS && kt < 0; base += 32) {
        const long long e = s_pexc[base + lane], n = s_psum[base + lane];
        const unsigned m = __ballot_sync(0xffffffffu, n > 0 && NI * (e + n) > start);
        if (m) kt = base + __ffs(m) - 1;
      }
      int bs = kt * bpt;
      long long preb = s_pexc[kt];
      for (;; ++bs) {
        long long t0;
        const long long n = (seq_len<LAYOUT>(p, bs, &t0) + PAGE - 1) / PAGE;
        if (NI * (preb + n) > start) break;
        preb += n;
      }
      int b = bs;
      long long tok0;
      int len = seq_len<LAYOUT>(p, b, &tok0);
      long long nb = (len + PAGE - 1) / PAGE;
      int hi = static_cast<int>((start - NI * preb) / nb);  // item head index (KV heads hi*HP ..)
      long long item_base = NI * preb + static_cast<long long>(hi) * nb;
      long long pos = start;

      // length of the next sequence, prefetched
      long long ntok0 = 0;
      int nlen = (b + 1 < p.B) ? seq_len<LAYOUT>(p, b + 1, &ntok0) : 0;
#ifdef FK_TRACE
      if (lane == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][17] = gtimer() + 0 * nlen;
      bool tr_f = true;
#endif

      while (alive && pos < end) {
        const long long seg_hi = min(end, item_base + nb);
        const int g0 = static_cast<int>(pos - item_base);
        const int g1 = static_cast<int>(seg_hi - item_base);
        const bool whole = (item_base >= start) && (item_base + nb <= end);
        const int seg = blockIdx.x + b * KVI + hi;
        const int c0 = static_cast<int>(item_base / per);
        const int nseg = static_cast<int>((item_base + nb - 1) / per) - c0 + 1;
        const int tbeg = g0 * PAGE;
        const int tend = min(g1 * PAGE, len);
        const int hcoord = item_kv<HP>(p, hi);  // first KV head of the item
#ifdef FK_TRACE
        unsigned long long tr_sw0 = gtimer();
#endif
        for (int tt = tbeg; tt < tend; tt += TT) {
          const int valid = min(TT, tend - tt);
#ifdef FK_TRACE
          const long long tc0 = clock64();
#endif
          if (!acquire()) {
            alive = false;
            break;
          }
          if (withhold) {
            withhold = false;
            advance();
            continue;
          }
#ifdef FK_TRACE
          const long long tc1 = clock64();
#endif
          const uint32_t sK = smem_u32(stages + stage * C::STAGE_BYTES);
          const uint32_t sV = sK + C::TILE_BYTES;
          const uint32_t fb = smem_u32(&full[stage]);
          int bad = 0;
          // chunk pairs load one KV head
          constexpr uint32_t nkv = CP ? 1u : static_cast<uint32_t>(HP);
          uint32_t bytes = 2u * C::TILE_BYTES;
          int phys = -1;
          if constexpr (LAYOUT == PAGED) {
            const int p0 = tt / PAGE;
            const int np = (valid + PAGE - 1) / PAGE;
            if (b != win_b || p0 < win_p0 || p0 + PPT > win_p0 + 32) {
              if (b == win_b && p0 == win_p0 + 32) {
                bt_cur = bt_nxt;
                win_p0 += 32;
              } else {
                win_b = b;
                win_p0 = p0;
                bt_cur = ld_bt(b, p0 + lane);
              }
              bt_nxt = ld_bt(b, win_p0 + 32 + lane);
            }
            phys = __shfl_sync(0xffffffffu, bt_cur, (p0 - win_p0) + (lane & (PPT - 1)));
            const bool okp = (lane < np) && phys >= 0 && phys < p.num_pages;
            const unsigned okm = __ballot_sync(0xffffffffu, okp) & ((1u << PPT) - 1u);
            bad = static_cast<int>(~okm & ((1u << np) - 1u));
            bytes = static_cast<uint32_t>(__popc(okm)) * 2u * nkv * C::PAGE_BYTES;
            if (lane == 0 && bad) atomicOr(&hdr->status, FK_STATUS_BAD_PAGE);
            if (!okp) phys = -1;
          }
#ifdef FK_TRACE
          const long long tc2 = clock64();
          if (tr_f && lane == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][18] = gtimer();
#endif
          int mqslot = 0;
          if (tt == tbeg) {
            if (!qacquire()) {
              alive = false;
              break;
            }
            mqslot = qslot;
            if (++qslot == C::QSLOTS) {
              qslot = 0;
              qphase ^= 1u;
            }
            uint32_t* qs = qstage + mqslot * QWORDS;
            if (q_async) {
              // the item's query rows of D * 2 bytes, 16 bytes per copy, into
              // 256-byte row slots
              const uint32_t qd = smem_u32(qs);
              const long long qb0 = static_cast<long long>(b) * p.q_sb;
              const int qes = (p.q_dtype == FK_DTYPE_E4M3) ? 1 : 2;  // Q bytes per element
              const int nch = D * qes / 16;                          // 16-byte copies per row
              const int nrow = item_rows<HP>(p, hi);
              for (int u = lane; u < nrow * nch; u += 32) {
                const int r = u / nch, c = u % nch;
                int hh, j;
                item_row<HP>(p, hi, r, hh, j);
                const int qh = item_q<HP>(p, hi, hh, j);
                cp_async16(qd + (hh * GPAD + j) * 256 + c * 16,
                           static_cast<const unsigned char*>(p.q) +
                               (qb0 + static_cast<long long>(qh) * p.q_sh) * qes + c * 16);
              }
              cp_async_mbar_arrive(fb);
            } else if constexpr (HP != 4) {  // (four-head items always take the cp.async path)
              // Q rows of the item -> the Q slot as packed MMA-type pairs,
              // from the registers prefetched one item ahead
              if (qpre_b != b || qpre_h != hi) q_prefetch(b, hi);
#pragma unroll
              for (int k = 0; k < QW; ++k) qs[lane + 32 * k] = q_pair_to_mma<C::BF16>(p, qpre[k], psq);
              // start fetching the next item's Q
              if (hi + 1 < KVI) q_prefetch(b, hi + 1);
              else if (b + 1 < p.B) q_prefetch(b + 1, 0);
              __threadfence_block();
            }
            __syncwarp();
          }
#ifdef FK_TRACE
          const long long tc3 = clock64();
          if (tr_f && lane == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][19] = gtimer();
#endif
          if (lane == 0) {
            Meta& mt = meta[stage];
            mt.b = b;
            mt.h = hi;
            mt.tok = tt;
            mt.valid = valid;
            mt.flags = (tt == tbeg ? F_FIRST : 0) | (tt + TT >= tend ? F_LAST : 0) | (whole ? F_WHOLE : 0);
            mt.seg = seg;
            mt.bad = bad;
            mt.c0 = c0;
            mt.nseg = nseg;
            mt.qslot = mqslot;
            mbar_arrive_expect_tx(fb, bytes);
          }
          armed |= 1u << stage;
          armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          __syncwarp();
          if constexpr (LAYOUT == PAGED) {
            if (phys >= 0) {
              // one box per page: 16 tokens x HP heads x D dims
              const uint32_t off = lane * (nkv * C::PAGE_BYTES);
              if constexpr (C::FP8) {
                tma_load_4d(sK + off, &p.tk, fb, 0, 0, hcoord, phys);
                tma_load_4d(sV + off, &p.tv, fb, 0, 0, hcoord, phys);
              } else {
                tma_load_5d(sK + off, &p.tk, fb, 0, 0, 0, hcoord, phys);
                tma_load_5d(sV + off, &p.tv, fb, 0, 0, 0, hcoord, phys);
              }
            }
          } else if (lane == 0) {
            // one box per stage: TT tokens x HP heads x D dims
            const int row = static_cast<int>(tok0 + tt);
            if constexpr (LAYOUT == VARLEN) {
              if constexpr (C::FP8) {
                tma_load_3d(sK, &p.tk, fb, 0, row, hcoord);
                tma_load_3d(sV, &p.tv, fb, 0, row, hcoord);
              } else {
                tma_load_4d(sK, &p.tk, fb, 0, row, 0, hcoord);
                tma_load_4d(sV, &p.tv, fb, 0, row, 0, hcoord);
              }
            } else {
              if constexpr (C::FP8) {
                tma_load_4d(sK, &p.tk, fb, 0, row, hcoord, b);
                tma_load_4d(sV, &p.tv, fb, 0, row, hcoord, b);
              } else {
                tma_load_5d(sK, &p.tk, fb, 0, row, 0, hcoord, b);
                tma_load_5d(sV, &p.tv, fb, 0, row, 0, hcoord, b);
              }
            }
          }
#ifdef FK_TRACE
          if (tt == tbeg && lane == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][5] += gtimer() - tr_sw0;
          if (tr_f && lane == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][20] = gtimer();
          tr_f = false;
          {
            const long long tc4 = clock64();
            tr_c[0] += tc2 - tc1;
            tr_c[1] += tc3 - tc2;
            tr_c[2] += tc4 - tc3;
            tr_c[3] += tc4 - tc0;
          }
#endif
          advance();
        }
        pos = seg_hi;
        if (pos >= end) break;
        if (++hi == KVI) {
          hi = 0;
          do {
            preb += nb;
            ++b;
            len = nlen;
            tok0 = ntok0;
            nb = (len + PAGE - 1) / PAGE;
            nlen = (b + 1 < p.B) ? seq_len<LAYOUT>(p, b + 1, &ntok0) : 0;
          } while (nb == 0 && b + 1 < p.B);
        }
        item_base = NI * preb + static_cast<long long>(hi) * nb;
      }
    }
#ifdef FK_TRACE
    if (lane == 0 && blockIdx.x < 4096)
      for (int i = 0; i < 4; ++i) g_trace[blockIdx.x][11 + i] = tr_c[i];
#endif
    // End-of-work marker.
    if (alive && acquire()) {
      if (lane == 0) {
        meta[stage].flags = F_END;
        mbar_arrive(smem_u32(&full[stage]));
      }
    } else if (lane == 0) {
      // A wait ran out: copies the consumers will never wait for may still be
      // in flight into this CTA's shared memory.  Let them land (each wait
      // bounded) before the CTA exits.
      for (int s2 = 0; s2 < C::STAGES; ++s2)
        if ((armed >> s2) & 1u) mbar_wait(smem_u32(&full[s2]), (armed_par >> s2) & 1u, p.wait_ns);
    }
    return;
  }

  if (warp > CWARPS) {
    // ================================================================ epilogue
    // Merge the consumer warps' states of each finished segment (per KV head:
    // its WPH warps); write whole items to `out`, split items to the
    // workspace, and let the CTA that completes a split item merge its
    // segments (CTA order: the result is deterministic) and re-arm its
    // arrival counter.
    const int et = threadIdx.x - (CWARPS + 1) * 32;  // 0 .. ETHREADS-1
    // Sequences of length 0 own no granules: CTA b % S writes their zero rows.
    for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
      long long t0;
      if (seq_len<LAYOUT>(p, b, &t0) == 0) {
        for (int qh = 0; qh < p.q_heads; ++qh)
          for (int d = et; d < D; d += ETHREADS)
            store_out(p, static_cast<long long>(b) * p.o_sb + static_cast<long long>(qh) * p.o_sh + d, 0.f);
      }
    }
    const float sv = (p.scale_v != nullptr) ? __ldg(p.scale_v) : 1.f;
    int eb = 0;
    uint32_t eph = 0;
    int it = 0;
    while (true) {
#ifdef FK_TRACE
      const unsigned long long te0 = gtimer();
#endif
      // Both epilogue warps act on the same outcome of the bounded wait (one
      // alone timing out must not leave the other in a named barrier).
      const bool wok = mbar_wait(smem_u32(&efull[eb]), eph, p.wait_ns);
      if (lane == 0) s_eok[it & 1][et >> 5] = wok ? 1 : 0;
      named_bar_sync(3, ETHREADS);
      bool eok = true;
#pragma unroll
      for (int w = 0; w < EWARPS; ++w) eok = eok && s_eok[it & 1][w] != 0;
      ++it;
      if (!eok) {
        if (et == 0) atomicOr(&hdr->status, FK_STATUS_TIMEOUT);
        break;
      }
#ifdef FK_TRACE
      const unsigned long long te1 = gtimer();
      if (et == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][23] += te1 - te0;
#endif
      const Meta mt = emeta[eb];
      if (mt.flags & F_END) {
#ifdef FK_TRACE
        if (et == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][27] = gtimer();
#endif
        break;
      }
      const EpiSlot& E = eslot[eb];
      const bool whole = (mt.flags & F_WHOLE) != 0;
      const long long item = static_cast<long long>(mt.b) * KVI + mt.h;
      const long long obase = static_cast<long long>(mt.b) * p.o_sb;
      // One unit per thread and round: query head hd of KV head hh (head
      // slot u / 8), dims (u % 8) * 4 + 32 k, k < D / 32 (a quarter warp reads
      // 128 contiguous bytes of the slot: no bank conflicts).
      const int nrow = item_rows<HP>(p, mt.h);
      for (int u = et; u < nrow * 8; u += ETHREADS) {
        const int r = u >> 3, d4 = (u & 7) * 4;
        int hh, hd;
        item_row<HP>(p, mt.h, r, hh, hd);
        float M = NEG_INF;
#pragma unroll
        for (int w = 0; w < WPH; ++w) M = fmaxf(M, E.cm[hh * WPH + w][hd]);
        float ew[WPH], L = 0.f;
#pragma unroll
        for (int w = 0; w < WPH; ++w) {
          ew[w] = (M == NEG_INF) ? 0.f : exp2f(E.cm[hh * WPH + w][hd] - M);
          L += ew[w] * E.cl[hh * WPH + w][hd];
        }
        float4 A[4];
#pragma unroll
        for (int k = 0; k < D / 32; ++k) A[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < WPH; ++w) {
#pragma unroll
          for (int k = 0; k < D / 32; ++k) {
            const float4 v = *reinterpret_cast<const float4*>(&E.cacc[hh * WPH + w][hd][d4 + 32 * k]);
            A[k].x += ew[w] * v.x;
            A[k].y += ew[w] * v.y;
            A[k].z += ew[w] * v.z;
            A[k].w += ew[w] * v.w;
          }
        }
        const int qh = item_q<HP>(p, mt.h, hh, hd);
        const int hs = hh * GPAD + hd;  // head slot in a segment record
        if (whole) {
          float e, Lf;
          sink_norm(L, M, p.s_aux, qh, &e, &Lf);
          const long long ob = obase + static_cast<long long>(qh) * p.o_sh + d4;
#pragma unroll
          for (int k = 0; k < D / 32; ++k) {
            store_out4(p, ob + 32 * k, norm_out(A[k].x, e, Lf, sv), norm_out(A[k].y, e, Lf, sv),
                       norm_out(A[k].z, e, Lf, sv), norm_out(A[k].w, e, Lf, sv));
          }
        } else {
          float4* dst = reinterpret_cast<float4*>(&ws_acc[(static_cast<long long>(mt.seg) * GSR + hs) * HEAD_DIM + d4]);
#pragma unroll
          for (int k = 0; k < D / 32; ++k) dst[8 * k] = A[k];
          if ((u & 7) == 0) ws_ml[static_cast<long long>(mt.seg) * GSR + hs] = make_float2(M, L);
        }
      }
      // the slot is consumed: give it back to the consumers
      mbar_arrive(smem_u32(&eempty[eb]));
#ifdef FK_TRACE
      if (et == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][22] += gtimer() - te1;
#endif
      if (++eb == C::NSLOT) {
        eb = 0;
        eph ^= 1u;
      }
      if (whole) continue;
      __threadfence();
      named_bar_sync(2, ETHREADS);
#ifdef FK_TRACE
      if (et == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][24] = gtimer();  // partial stored, before the atomic
#endif
      if (et == 0) s_last = (atomicAdd(&cnt[item], 1) == mt.nseg - 1) ? 1 : 0;
#ifdef FK_TRACE
      if (et == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][25] = gtimer();  // atomic returned
#endif
      named_bar_sync(2, ETHREADS);
      if (!s_last) continue;
      __threadfence();
      // All head slots in parallel: unit u = (slot u / KD, dims (u % KD) * 16
      // .. +16); each thread merges its units with 4 segments' loads in flight.
      for (int u = et; u < nrow * KD; u += ETHREADS) {
        const int r = u / KD, d0 = (u % KD) * 16;
        int hh, hd;
        item_row<HP>(p, mt.h, r, hh, hd);
        const int hs = hh * GPAD + hd;
        float M = NEG_INF, L = 0.f;
        float A[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) A[i] = 0.f;
        for (int c = 0; c < mt.nseg; c += 4) {
          float2 ml[4];
          float4 av[4][4];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const long long sg = item + mt.c0 + c + v;
            const bool ok = c + v < mt.nseg;
            ml[v] = ok ? __ldcg(&ws_ml[sg * GSR + hs]) : make_float2(NEG_INF, 0.f);
            const float4* src = reinterpret_cast<const float4*>(&ws_acc[(sg * GSR + hs) * HEAD_DIM + d0]);
#pragma unroll
            for (int i = 0; i < 4; ++i) av[v][i] = ok ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
          float Mn = M;
#pragma unroll
          for (int v = 0; v < 4; ++v) Mn = fmaxf(Mn, ml[v].x);
          if (Mn == NEG_INF) continue;
          const float sc = exp2f(M - Mn);
          L *= sc;
#pragma unroll
          for (int i = 0; i < 16; ++i) A[i] *= sc;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const float e = exp2f(ml[v].x - Mn);
            L += e * ml[v].y;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              A[4 * i + 0] += e * av[v][i].x;
              A[4 * i + 1] += e * av[v][i].y;
              A[4 * i + 2] += e * av[v][i].z;
              A[4 * i + 3] += e * av[v][i].w;
            }
          }
          M = Mn;
        }
        const int qh = item_q<HP>(p, mt.h, hh, hd);
        const long long ob = obase + static_cast<long long>(qh) * p.o_sh + d0;
        float e, Lf;
        sink_norm(L, M, p.s_aux, qh, &e, &Lf);
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          store_out4(p, ob + i, norm_out(A[i], e, Lf, sv), norm_out(A[i + 1], e, Lf, sv),
                     norm_out(A[i + 2], e, Lf, sv), norm_out(A[i + 3], e, Lf, sv));
      }
      if (et == 0) cnt[item] = 0;
#ifdef FK_TRACE
      if (et == 0 && blockIdx.x < 4096) {
        g_trace[blockIdx.x][26] = gtimer();  // merge done
        g_trace[blockIdx.x][28] += 1;
        g_trace[blockIdx.x][29] = mt.nseg;
      }
#endif
    }
#ifdef FK_TRACE
    if (et == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][9] = gtimer();
#endif
    return;
  }

  // ================================================================ consumers
  constexpr bool FP8 = C::FP8;
  constexpr bool MBF16 = C::BF16;  // MMA element type (FP8 KV computes in f16)
  const int g = lane >> 2;
  const int t = lane & 3;
  const int hh = warp / WPH;            // head slot of the item this warp serves
  const int hk = CP ? 0 : hh;            // its KV head's tile in the stage
  const int r0 = (warp % WPH) * 16;      // its 16 rows of that head's tile
  const float sk = (p.scale_k != nullptr) ? __ldg(p.scale_k) : 1.f;
  // Q staged raw by cp.async but not of the MMA type: convert on load
  const float qscale = (QC && p.scale_q != nullptr) ? __ldg(p.scale_q) : 1.f;
  const float qk_scale = rsqrtf(static_cast<float>(D)) * LOG2E * sk;

  float m[2], l[2], acc[KD][4];
  uint32_t qb[KD][2];
  int stage = 0;
  uint32_t phase = 0;
  int eb = 0;            // epilogue slot
  uint32_t ephase = 0;

  // Thread-constant shared-memory offsets.
  const int lr = lane & 7, lq = lane >> 3;
  // 16-bit path: ldmatrix row addresses.
  const int krow = r0 + lr + ((lq & 1) << 3);
  const int vrow = r0 + lr + ((lq >> 1) << 3);
  // FP8 path: logical token g <-> tile row prow (and prow + 8); V rows
  // r0 + t + 4(r&1) + 8(r>>1); V dim chunk cg.
  const int prow = r0 + (g >> 1) + ((g & 1) << 2);
  const int cg = (g >> 1) | ((g & 1) << 2);

  while (true) {
#ifdef FK_TRACE
    const unsigned long long tw0 = gtimer();
#endif
    if (!mbar_wait(smem_u32(&full[stage]), phase, p.wait_ns)) {
      if (lane == 0) atomicOr(&hdr->status, FK_STATUS_TIMEOUT);
      break;
    }
    const Meta mt = meta[stage];
    if (mt.flags & F_END) {
      // tell the epilogue warps to finish
      if (mbar_wait(smem_u32(&eempty[eb]), ephase ^ 1u, p.wait_ns)) {
        if (warp == 0 && lane == 0) emeta[eb].flags = F_END;
        mbar_arrive(smem_u32(&efull[eb]));
      } else if (lane == 0) {
        atomicOr(&hdr->status, FK_STATUS_TIMEOUT);
      }
      break;
    }
#ifdef FK_TRACE
    if (threadIdx.x == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][(mt.flags & F_FIRST) ? 7 : 8] += gtimer() - tw0;
    if (tr_first && threadIdx.x == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][1] = gtimer();
    tr_first = false;
    ++tr_ntile;
    if (mt.flags & F_LAST) ++tr_nseg;
#endif

    if (mt.flags & F_FIRST) {
      m[0] = m[1] = NEG_INF;
      l[0] = l[1] = 0.f;
#pragma unroll
      for (int i = 0; i < KD; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
      // the producer staged this item's Q rows (zero-padded to 8 heads) next
      // to the segment's first tile: raw rows (cp.async) or MMA-type pairs
      const uint32_t* qrow = qstage + mt.qslot * QWORDS + hh * (GPAD * 64) + g * 64;
#pragma unroll
      for (int j = 0; j < KD; ++j) {
        int d0, d1;
        if constexpr (FP8) {
          d0 = (j < 4) ? (16 * t + 4 * j) : (64 + 16 * t + 4 * (j - 4));
          d1 = d0 + 2;
        } else {
          d0 = 16 * j + 2 * t;
          d1 = d0 + 8;
        }
        if constexpr (!QC) {
          qb[j][0] = qrow[d0 >> 1];
          qb[j][1] = qrow[d1 >> 1];
        } else if (p.q_dtype == FK_DTYPE_E4M3) {  // raw bytes: pair (d, d+1) at byte d
          const unsigned char* qbytes = reinterpret_cast<const unsigned char*>(qrow);
          qb[j][0] = q_pair_to_mma<MBF16>(p, *reinterpret_cast<const unsigned short*>(qbytes + d0), qscale);
          qb[j][1] = q_pair_to_mma<MBF16>(p, *reinterpret_cast<const unsigned short*>(qbytes + d1), qscale);
        } else {  // raw 16-bit pairs of the other 16-bit type
          qb[j][0] = q_pair_to_mma<MBF16>(p, qrow[d0 >> 1], qscale);
          qb[j][1] = q_pair_to_mma<MBF16>(p, qrow[d1 >> 1], qscale);
        }
      }
      // this warp holds its Q rows in registers: release the Q slot
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&qempty[mt.qslot]));
    }

    // Blocks of 16 rows of this warp in the stage (two at D = 64).
    constexpr int NBLK = C::TILE / 64;
#ifdef FK_EXP_NOMATH
    if (false)
#endif
#pragma unroll
    for (int blk = 0; blk < NBLK; ++blk) {
      const int bo = blk * (WPH * 16);  // row offset of the block
      const int r0b = r0 + bo;
      if (r0b >= mt.valid) break;
      const uint32_t sK = smem_u32(stages + stage * C::STAGE_BYTES);
      const uint32_t sV = sK + C::TILE_BYTES;
      const bool partial = (r0b + 16 > mt.valid) || (mt.bad != 0);
      auto tok_ok = [&](int row) -> bool { return row < mt.valid && !((mt.bad >> (row >> 4)) & 1); };

      // ---- S^T = K Q^T : 16 tokens x 8 heads
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      float s2[4] = {0.f, 0.f, 0.f, 0.f};  // odd k-steps: two independent MMA chains
      int rowA, rowB;
      // e4m3: this block's V rows are loaded up front, so that the loads are
      // in flight while QK^T and the softmax run (PV waits only on P)
      uint4 vx[FP8 ? 4 : 1];
      if constexpr (FP8) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int row = r0b + t + 4 * (r & 1) + 8 * (r >> 1);
          vx[r] = lds128(sV + TL::row_off(hk, row) + ((cg ^ (row & 7)) << 4));
        }
      }
      if constexpr (FP8) {
        rowA = (prow + bo);
        rowB = (prow + bo) + 8;
        const int sw = (prow + bo) & 7;
        const uint32_t ra = sK + TL::row_off(hk, (prow + bo)), rb = ra + 8 * 128;
        const uint4 alo = lds128(ra + ((t ^ sw) << 4));
        const uint4 ahi = lds128(ra + (((t + 4) ^ sw) << 4));
        const uint4 blo = lds128(rb + ((t ^ sw) << 4));
        const uint4 bhi = lds128(rb + (((t + 4) ^ sw) << 4));
        const uint32_t wa[8] = {alo.x, alo.y, alo.z, alo.w, ahi.x, ahi.y, ahi.z, ahi.w};
        const uint32_t wb[8] = {blo.x, blo.y, blo.z, blo.w, bhi.x, bhi.y, bhi.z, bhi.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t a0, a1, a2, a3;
          e4m3x4_to_f16x2x2(wa[j], a0, a2);
          e4m3x4_to_f16x2x2(wb[j], a1, a3);
          if (j & 1) mma16816<false>(s2, a0, a1, a2, a3, qb[j][0], qb[j][1]);
          else mma16816<false>(s, a0, a1, a2, a3, qb[j][0], qb[j][1]);
        }
      } else {
        rowA = r0b + g;
        rowB = r0b + g + 8;
        const uint32_t kb = sK + TL::row_off(hk, (krow + bo));
        const int ksw = (krow + bo) & 7;
#pragma unroll
        for (int j = 0; j < KD; ++j) {
          const int c = ((j & 3) << 1) + (lq >> 1);
          uint32_t a0, a1, a2, a3;
          ldsm_x4(kb + (j >> 2) * TL::HALF_STRIDE + ((c ^ ksw) << 4), a0, a1, a2, a3);
          if (j & 1) mma16816<MBF16>(s2, a0, a1, a2, a3, qb[j][0], qb[j][1]);
          else mma16816<MBF16>(s, a0, a1, a2, a3, qb[j][0], qb[j][1]);
        }
      }

#pragma unroll
      for (int i = 0; i < 4; ++i) s[i] += s2[i];
      // ---- online softmax (log2 domain), heads 2t and 2t+1
      bool okA = true, okB = true;
      if (partial) {
        okA = tok_ok(rowA);
        okB = tok_ok(rowB);
      }
      const float x0 = okA ? s[0] * qk_scale : NEG_INF;
      const float x1 = okA ? s[1] * qk_scale : NEG_INF;
      const float x2 = okB ? s[2] * qk_scale : NEG_INF;
      const float x3 = okB ? s[3] * qk_scale : NEG_INF;
      // The running max moves only when a logit exceeds it by more than
      // LAZY_MAX (log2 units): the warp-wide max reduction and the rescale
      // are skipped otherwise, and P = 2^(x - m) stays below 2^LAZY_MAX
      // (well inside f16 range).  Any reference m gives the same softmax once
      // acc and l are normalised together; only the rounding differs.
      constexpr float LAZY_MAX = MBF16 ? 0.f : LAZY_MAX_F16;
      float al0 = 1.f, al1 = 1.f;
      const bool grow = fmaxf(x0, x2) > m[0] + LAZY_MAX || fmaxf(x1, x3) > m[1] + LAZY_MAX;
      if (__any_sync(0xffffffffu, grow)) {
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
        al0 = exp2f(m[0] - ((mn0 == NEG_INF) ? 0.f : mn0));
        al1 = exp2f(m[1] - ((mn1 == NEG_INF) ? 0.f : mn1));
        m[0] = mn0;
        m[1] = mn1;
#pragma unroll
        for (int i = 0; i < KD; ++i) {
          acc[i][0] *= al0;
          acc[i][1] *= al1;
          acc[i][2] *= al0;
          acc[i][3] *= al1;
        }
      }
      const float b0s = (m[0] == NEG_INF) ? 0.f : m[0];
      const float b1s = (m[1] == NEG_INF) ? 0.f : m[1];
      const float p0 = exp2f(x0 - b0s), p1 = exp2f(x1 - b1s);
      const float p2 = exp2f(x2 - b0s), p3 = exp2f(x3 - b1s);
      l[0] = l[0] * al0 + (p0 + p2);
      l[1] = l[1] * al1 + (p1 + p3);
      // P^T as the B operand: transpose the 8x8 (token x head) blocks.
      const uint32_t pb0 = movmatrix_t(pack2<MBF16>(p0, p1));
      const uint32_t pb1 = movmatrix_t(pack2<MBF16>(p2, p3));

      // ---- O^T += V^T P^T : D dims x 8 heads
      if constexpr (FP8) {
        uint4 x[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int row = r0b + t + 4 * (r & 1) + 8 * (r >> 1);
          x[r] = vx[r];
          if (partial && !tok_ok(row)) x[r] = make_uint4(0u, 0u, 0u, 0u);
        }
        const uint32_t w0[4] = {x[0].x, x[0].y, x[0].z, x[0].w};
        const uint32_t w1[4] = {x[1].x, x[1].y, x[1].z, x[1].w};
        const uint32_t w2[4] = {x[2].x, x[2].y, x[2].z, x[2].w};
        const uint32_t w3[4] = {x[3].x, x[3].y, x[3].z, x[3].w};
#pragma unroll
        for (int i = 0; i < KD; ++i) {
          const uint32_t sel = (i & 1) ? 0x7362u : 0x5140u;
          const uint32_t u01 = __byte_perm(w0[i >> 1], w1[i >> 1], sel);
          const uint32_t u89 = __byte_perm(w2[i >> 1], w3[i >> 1], sel);
          uint32_t a0, a1, a2, a3;
          e4m3x4_to_f16x2x2(u01, a0, a1);
          e4m3x4_to_f16x2x2(u89, a2, a3);
          mma16816<false>(acc[i], a0, a1, a2, a3, pb0, pb1);
        }
      } else {
        uint32_t mk01 = 0xffffffffu, mk89 = 0xffffffffu;
        if (partial) {
          const int tk = r0b + 2 * t;
          mk01 = (tok_ok(tk) ? 0x0000ffffu : 0u) | (tok_ok(tk + 1) ? 0xffff0000u : 0u);
          mk89 = (tok_ok(tk + 8) ? 0x0000ffffu : 0u) | (tok_ok(tk + 9) ? 0xffff0000u : 0u);
        }
        const uint32_t vb = sV + TL::row_off(hk, (vrow + bo));
        const int vsw = (vrow + bo) & 7;
#pragma unroll
        for (int i = 0; i < KD; ++i) {
          const int c = ((2 * i) & 7) + (lq & 1);
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(vb + (i >> 2) * TL::HALF_STRIDE + ((c ^ vsw) << 4), a0, a1, a2, a3);
          mma16816<MBF16>(acc[i], a0 & mk01, a1 & mk01, a2 & mk89, a3 & mk89, pb0, pb1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty[stage]));

    if (mt.flags & F_LAST) {
      // ---- hand this segment's state to the epilogue warps and go on
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        l[0] += __shfl_xor_sync(0xffffffffu, l[0], o);
        l[1] += __shfl_xor_sync(0xffffffffu, l[1], o);
      }
#ifdef FK_TRACE
      const unsigned long long tq = gtimer();
#endif
      const bool eok = mbar_wait(smem_u32(&eempty[eb]), ephase ^ 1u, p.wait_ns);
#ifdef FK_TRACE
      if (threadIdx.x == 0 && blockIdx.x < 4096) g_trace[blockIdx.x][21] += gtimer() - tq;
#endif
      if (!eok) {
        if (lane == 0) atomicOr(&hdr->status, FK_STATUS_TIMEOUT);
        break;
      }
      EpiSlot& E = eslot[eb];
      if (g == 0) {
        E.cm[warp][2 * t] = m[0];
        E.cm[warp][2 * t + 1] = m[1];
        E.cl[warp][2 * t] = l[0];
        E.cl[warp][2 * t + 1] = l[1];
      }
#pragma unroll
      for (int i = 0; i < KD; ++i) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int d = FP8 ? (16 * cg + 2 * i + r) : (16 * i + g + 8 * r);
#pragma unroll
          for (int j = 0; j < 2; ++j) E.cacc[warp][2 * t + j][d] = acc[i][2 * r + j];
        }
      }
      if (warp == 0 && lane == 0) emeta[eb] = mt;
      mbar_arrive(smem_u32(&efull[eb]));
      if (++eb == C::NSLOT) {
        eb = 0;
        ephase ^= 1u;
      }
    }
    if (++stage == C::STAGES) {
      stage = 0;
      phase ^= 1u;
    }
  }
#ifdef FK_TRACE
  if (threadIdx.x == 0 && blockIdx.x < 4096) {
    g_trace[blockIdx.x][2] = gtimer();
    g_trace[blockIdx.x][3] = tr_nseg;
    g_trace[blockIdx.x][4] = tr_ntile;

  }
#endif
}

}  // namespace fk

// Every kernel instantiation the host side launches, per KV element type:
// X(KV, LAYOUT, HP, D, CP, QC).  Each list is explicitly instantiated in its
// own translation unit (fk_kernels_<type>.cu) so that the three compile in
// parallel; fk_decode.cu declares them extern.
#define FK_KERNELS_LAYOUTS(X, KVT, H, DD, CC, QQ) \
  X(KVT, 0, H, DD, CC, QQ) X(KVT, 1, H, DD, CC, QQ) X(KVT, 2, H, DD, CC, QQ)
#define FK_KERNELS_HP(X, KVT, DD, QQ)                                                        \
  FK_KERNELS_LAYOUTS(X, KVT, 1, DD, false, QQ) FK_KERNELS_LAYOUTS(X, KVT, 2, DD, false, QQ) \
  FK_KERNELS_LAYOUTS(X, KVT, 2, DD, true, QQ)
#define FK_KERNELS_F16(X) FK_KERNELS_HP(X, FK_DTYPE_F16, 64, false) FK_KERNELS_HP(X, FK_DTYPE_F16, 128, false)
#define FK_KERNELS_BF16(X) FK_KERNELS_HP(X, FK_DTYPE_BF16, 64, false) FK_KERNELS_HP(X, FK_DTYPE_BF16, 128, false)
#define FK_KERNELS_E4M3(X)                                                                                  \
  FK_KERNELS_HP(X, FK_DTYPE_E4M3, 128, false) FK_KERNELS_HP(X, FK_DTYPE_E4M3, 128, true)                   \
  FK_KERNELS_LAYOUTS(X, FK_DTYPE_E4M3, 4, 128, false, false) FK_KERNELS_LAYOUTS(X, FK_DTYPE_E4M3, 4, 128, false, true)
#define FK_KERNEL_DECL(KVT, L, H, DD, CC, QQ) \
  extern template __global__ void fk::decode_split_kernel<KVT, L, H, DD, CC, QQ>(const __grid_constant__ fk::Params);
#define FK_KERNEL_INST(KVT, L, H, DD, CC, QQ) \
  template __global__ void fk::decode_split_kernel<KVT, L, H, DD, CC, QQ>(const __grid_constant__ fk::Params);
