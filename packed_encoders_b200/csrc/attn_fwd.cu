// Packed variable-length attention for B200 (sm_100a): a device tile-schedule builder and a
// persistent, warp-specialised tcgen05 forward kernel, behind the C ABI of pe_b200_attn.h.
//
// Work decomposition (packed_encoders/_kernels/triton_packed_attention.py:72-143 computes the
// same function with one program per (sequence, head, 16/64-row query block)):
//   * a WORK ITEM is one 128-row query tile. Sequences longer than 128 tokens get one item per
//     128-row block; runs of consecutive short sequences (query and key spans <= 128 each) are
//     packed greedily into ONE item whose key tile is block-diagonal: each row reads only the
//     keys of its own sequence (the short-sequence variant);
//   * items are ordered by cost (number of key tiles), longest first, and a UNIT is
//     (item, head). CTA b of the persistent grid takes units b, b + grid, b + 2*grid, ...
//   * per unit the key range is the union of the rows' allowed keys (window / causal), walked
//     in key tiles of BN tokens; rows mask keys outside their own band.
//
// Roles inside one CTA (192 threads):
//   warp 0        TMA producer: Q tile (double-buffered across units), K/V key tiles (rings),
//                 and each unit's row slot (header + every row's allowed key interval)
//   warp 1        MMA issuer: S = Q K^T (SS form) into two (or three) TMEM S buffers, then
//                 O += P V with P read from TMEM (TS form), one or two key tiles behind QK;
//                 units taken from the row slots; TMEM allocator
//   warps 2..5    softmax + epilogue: one query row per thread (TMEM lane), exp2 online
//                 softmax with fp32 row max / sum, bf16 P written back over S, O rescaled in
//                 TMEM only when the running max grows by more than 2^8, final O / l -> bf16
// Passes next to it: rope_pass_kernel (rotary tables, before the attention) and
// gate_pass_kernel (output gate, after it).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/pe_b200_attn.h"
#include "sm100_ptx.cuh"

namespace pe_b200 {

constexpr int kTileM = 128;               // query rows per item / TMEM lanes
constexpr int kHeaderBytes = 256;         // workspace header: n_items, error word
// L2 policies of the TMA copies: Q tiles are read once (evict first); K/V tiles are re-read by
// every query block of their sequence (0 normal, 1 evict last). Output rows are written with
// streaming stores.
constexpr bool kQEvictFirst = true;
constexpr int kKVPolicy = 0;
constexpr bool kStreamOut = true;

constexpr int kCostBuckets = 1024;        // LPT ordering buckets (cost clamped)
constexpr int kBuilderThreads = 1024;
constexpr float kRescaleThreshold = 8.0f; // log2 units: rescale O only when the max grows > 2^8

struct WorkItem {
  int seq_first;  // first sequence of the item
  int seq_count;  // 1 for a block of one sequence; >= 1 for a packed run of short sequences
  int q_block;    // 128-row block index inside seq_first (0 for packed runs)
  int cost;       // key tiles
};

struct WsHeader {
  int n_items;
  int error;
};

struct SchedParams {
  const int32_t* cu_q;
  const int32_t* cu_k;
  int n_seq;
  int total_q;
  int total_k;
  int window_left;   // -1 unbounded
  int window_right;  // -1 unbounded; 0 when causal
  int block_n;       // key tile
  int capacity;      // items the workspace holds
  WsHeader* header;
  WorkItem* items;
};

struct AttnParams {
  const int32_t* cu_q;
  const int32_t* cu_k;
  int heads;
  int group;  // heads / kv_heads
  int total_q;
  __nv_bfloat16* out;
  long long o_tok;
  long long o_head;
  float* lse;
  float scale_log2;
  int window_left;
  int window_right;
  const WsHeader* header;
  const WorkItem* items;
  int* err;
  const __nv_bfloat16* gate;  // optional output gate [total_q, heads, D]
  long long g_tok;
  long long g_head;
  int kv_major;  // unit order (unit_coords)
  // q, k, v as the tensor maps read them; only the non-finite row rewrite reads them through these.
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  long long q_tok, q_head, k_tok, k_head, v_tok, v_head;
};

// ---------------------------------------------------------------------------------------------
// Key range of a block of one sequence (shared by the builder's cost and the kernel's walk).
// Query rows [qb*128, qb*128 + nq) of a segment with lq queries and lk keys; queries sit at key
// position row + (lk - lq) (end-aligned). Returns [lo, hi) in key-local positions.
__host__ __device__ __forceinline__ void block_key_range(int qb, int nq, int lq, int lk, int wl, int wr, int& lo,
                                                         int& hi) {
  int shift = lk - lq;
  int p0 = qb * kTileM + shift;
  int p1 = qb * kTileM + nq - 1 + shift;
  lo = wl >= 0 ? max(0, p0 - wl) : 0;
  hi = wr >= 0 ? min(lk, p1 + wr + 1) : lk;
  if (hi < lo) hi = lo;
}

__device__ __forceinline__ int cost_bucket(int cost) { return min(max(cost, 0), kCostBuckets - 1); }

// Greedy walk over sequences [lo, hi): emits items in order through
// `emit(item, index_in_group, group_size, group_cost)`. The query blocks of one long sequence
// form a group that is placed contiguously in the schedule (ordered by the group's largest
// item cost), so CTAs running at the same time share that sequence's K/V in L2; a packed
// block of short sequences is a group of one.
template <class Emit>
__device__ void walk_sequences(const SchedParams& p, int lo, int hi, Emit emit) {
  int first = -1, count = 0, span_q = 0, span_k = 0;
  auto close = [&]() {
    if (first >= 0 && span_q > 0) {
      WorkItem it{first, count, 0, (span_k + p.block_n - 1) / p.block_n};
      emit(it, 0, 1, it.cost);
    }
    first = -1;
    count = 0;
    span_q = span_k = 0;
  };
  for (int s = lo; s < hi; ++s) {
    int lq = p.cu_q[s + 1] - p.cu_q[s];
    int lk = p.cu_k[s + 1] - p.cu_k[s];
    if (lq <= 0) {  // no query rows: keep contiguity of an open run if its keys fit
      if (first >= 0 && span_k + lk <= kTileM) {
        ++count;
        span_k += lk;
      } else {
        close();
      }
      continue;
    }
    if (lq > kTileM || lk > kTileM) {  // a long sequence: one item per 128-row query block
      close();
      const int nblk = (lq + kTileM - 1) / kTileM;
      auto item_of = [&](int qb) {
        const int nq = min(kTileM, lq - qb * kTileM);
        int klo, khi;
        block_key_range(qb, nq, lq, lk, p.window_left, p.window_right, klo, khi);
        return WorkItem{s, 1, qb, (khi - klo + p.block_n - 1) / p.block_n};
      };
      int group_cost = 0;
      for (int qb = 0; qb < nblk; ++qb) group_cost = max(group_cost, item_of(qb).cost);
      for (int qb = 0; qb < nblk; ++qb) emit(item_of(qb), qb, nblk, group_cost);
      continue;
    }
    if (first >= 0 && span_q + lq <= kTileM && span_k + lk <= kTileM) {
      ++count;
      span_q += lq;
      span_k += lk;
    } else {
      close();
      first = s;
      count = 1;
      span_q = lq;
      span_k = lk;
    }
  }
  close();
}

__device__ int block_exclusive_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tmp[w] = x;
  __syncthreads();
  if (w == 0) {
    int s = lane < nw ? tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    tmp[lane] = s;
  }
  __syncthreads();
  int off = (w > 0 ? tmp[w - 1] : 0) + x - v;
  *total = tmp[nw - 1];
  __syncthreads();
  return off;
}

// One CTA builds the whole schedule: validate segments, greedy-pack per thread chunk, count
// items per cost bucket, order buckets longest-first, scatter.
__global__ void __launch_bounds__(kBuilderThreads) schedule_kernel(SchedParams p) {
  __shared__ int hist[kCostBuckets];
  __shared__ int cursor[kCostBuckets];
  __shared__ int tmp[32];
  __shared__ int bad;
  const int tid = threadIdx.x;
  for (int b = tid; b < kCostBuckets; b += blockDim.x) hist[b] = 0;
  if (tid == 0) {
    bad = 0;
    p.header->error = 0;  // the header is this thread's alone; n_items is written at the end
  }
  __syncthreads();
  for (int s = tid; s < p.n_seq; s += blockDim.x) {
    int q0 = p.cu_q[s], q1 = p.cu_q[s + 1], k0 = p.cu_k[s], k1 = p.cu_k[s + 1];
    bool ok = q0 <= q1 && k0 <= k1 && (q1 - q0) <= (k1 - k0) && q0 >= 0 && k0 >= 0 && q1 <= p.total_q &&
              k1 <= p.total_k;
    if (s == 0) ok = ok && q0 == 0 && k0 == 0;
    if (s == p.n_seq - 1) ok = ok && q1 == p.total_q && k1 == p.total_k;
    if (!ok) atomicOr(&bad, 1);
  }
  __syncthreads();
  if (bad) {
    if (tid == 0) {
      p.header->n_items = 0;
      atomicOr(&p.header->error, kErrBadSegments);
    }
    return;
  }
  const int chunk = (p.n_seq + blockDim.x - 1) / blockDim.x;
  const int lo = min(p.n_seq, tid * chunk), hi = min(p.n_seq, lo + chunk);
  walk_sequences(p, lo, hi, [&](const WorkItem&, int, int, int group_cost) {
    atomicAdd(&hist[cost_bucket(group_cost)], 1);
  });
  __syncthreads();
  int total = 0;
  for (int base = 0; base < kCostBuckets; base += blockDim.x) {  // blockDim == kCostBuckets
    int b = kCostBuckets - 1 - (base + tid);
    int off = block_exclusive_scan(b >= 0 ? hist[b] : 0, tmp, &total);
    if (b >= 0) cursor[b] = off;
  }
  __syncthreads();
  int group_base = 0;
  walk_sequences(p, lo, hi, [&](const WorkItem& it, int index, int group_size, int group_cost) {
    if (index == 0) group_base = atomicAdd(&cursor[cost_bucket(group_cost)], group_size);
    const int pos = group_base + index;
    if (pos < p.capacity) p.items[pos] = it;
  });
  if (tid == 0) {
    if (total > p.capacity) atomicOr(&p.header->error, kErrScheduleOverflow);
    p.header->n_items = min(total, p.capacity);
  }
}

__global__ void clear_header_kernel(WsHeader* h) {
  h->n_items = 0;
  h->error = 0;
}

// ---------------------------------------------------------------------------------------------
// Attention kernel configuration.
//   D   head_dim;  BN key-tile rows;  ST / VST K / V ring stages (K is released after QK, V after
//       P.V, and K runs one key tile ahead of V);  QB Q-tile buffers;
//   NS  S buffers in TMEM (2: QK of the next key tile overlaps the softmax of this one;
//       3: QK runs two key tiles ahead of P.V, measured faster for windowed layers and batches
//       of short sequences, whose units are a few key tiles long; 1: a single S, so several
//       CTAs share an SM and overlap each other);
//   CPS CTAs per SM the configuration is sized for (TMEM columns, shared memory, registers).
//   POLY of every 16 exp2 pairs evaluated by a cubic on the FMA pipe instead of MUFU.
//   PASS S columns a softmax thread holds in registers at once (0: min(BN, 64)); a row wider
//        than PASS is re-read from TMEM for the exp pass.
//   TMA_OUT windowed-layer epilogue through one TMA store per warp; GATE output gate fused into
//        the epilogue; STAGE epilogue rows staged through shared memory (head_dim 64).
template <int D_, int BN_, int ST_, int VST_, int QB_, int NS_, int CPS_, int POLY_ = 0, int PASS_ = 0,
          bool TMA_OUT_ = false, bool GATE_ = false, bool STAGE_ = true, bool QTM_ = false>
struct Cfg {
  static constexpr bool kGate = GATE_;  // output gate fused into the epilogue (calls with a gate)
  static constexpr int D = D_, BN = BN_, ST = ST_, VST = VST_, QB = QB_, NS = NS_, CPS = CPS_, POLY = POLY_;
  static constexpr int kPass = PASS_ > 0 ? PASS_ : (BN < 64 ? BN : 64);
  static constexpr int kThreads = 192;
  // Registers per thread that let CPS CTAs share an SM's 64K (allocated in steps of 8).
  static constexpr int kMaxRegs = (65536 / (kThreads * CPS)) / 8 * 8 > 255 ? 255 : (65536 / (kThreads * CPS)) / 8 * 8;
  static constexpr int kPanels = D / 64;                 // 64-element (128-byte) column panels
  // MMAs go in groups of four (one 64-deep slice) from one lane elected once, QK and P.V
  // (config 5, head_dim 256: -4 %; head_dim 64: config 3 local -3 %, config 2 -1 %).
  static constexpr int kQPanelBytes = kTileM * 128;      // one panel of a 128-row tile
  static constexpr int kKVPanelBytes = BN * 128;
  static constexpr int kQBytes = kPanels * kQPanelBytes;
  static constexpr int kKVBytes = kPanels * kKVPanelBytes;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + QB * kQBytes;
  static constexpr int kOffV = kOffK + ST * kKVBytes;
  static constexpr int kOffBar = kOffV + VST * kKVBytes;
  // barriers: k_full[ST] k_empty[ST] v_full[VST] v_empty[VST] q_full[QB] q_empty[QB] s_full[NS] p_full[NS]
  //           o_full row_empty[QB]
  static constexpr int kNumBars = 2 * ST + 2 * VST + 3 * QB + 2 * NS + 1;
  static constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
  // Epilogue staging (2 KB per softmax warp) so output rows leave as coalesced 128-byte lines;
  // only where shared memory allows (head_dim 64).
  static constexpr bool kStageOut = STAGE_ && D == 64 && CPS > 1;
  // TMA_OUT: each warp's 32 staged rows leave through one TMA store (4 KB per warp, 128-byte
  // swizzle: 16-byte chunk c of row r at r*128 + (c ^ r % 8)*16). Measured faster for windowed
  // layers (config 3 local -9 %) and slower for global layers and query batches (+2 % / +5 %),
  // so it is chosen per attention kind.
  static constexpr bool kTmaOut = TMA_OUT_ && kStageOut;
  static constexpr int kStageAlign = kTmaOut ? 1024 : 128;  // the 128-byte swizzle needs 1 KB
  static constexpr int kOffStage = (kOffTmemSlot + 16 + kStageAlign - 1) & ~(kStageAlign - 1);
  static constexpr int kStageBytes = kTmaOut ? 4 * 4096 : kStageOut ? 4 * 2048 : 0;
  // Per Q buffer: the unit's header (UnitInfo fields) and every row's allowed key interval,
  // written by the producer so the softmax warps read no schedule data from global memory.
  static constexpr int kRowSlotBytes = 64 + kTileM * 8;
  static constexpr int kOffRows = kOffStage + kStageBytes;
  static constexpr int kSmemBytes = kOffRows + QB * kRowSlotBytes + 1024;  // + align slack
  static constexpr uint32_t kColO = NS * BN;
  // QTM: the unit's Q tile is copied into TMEM (tcgen05.cp, D / 2 columns after O) and the QK
  // MMAs read it from there, so each of their k-steps reads only the K tile from shared memory.
  static constexpr bool kQTmem = QTM_;
  static constexpr uint32_t kColQ = kColO + D;
  static constexpr uint32_t kTmemUsed = kColQ + (kQTmem ? D / 2 : 0);
  static constexpr uint32_t kTmemCols = (kTmemUsed <= 128) ? 128 : (kTmemUsed <= 256) ? 256 : 512;
  static_assert(NS * BN <= (int)kColO && kTmemUsed <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
  // CPS CTAs must fit one SM together: 228 KB of shared memory (1 KB of it reserved per CTA).
  static_assert((kSmemBytes + 1024) * CPS <= 228 * 1024, "shared memory of CPS CTAs per SM");
  static_assert(BN % 64 == 0 && D % 64 == 0 && BN % kPass == 0 && kPass % 32 == 0, "tile shape");
  static_assert(kTmemCols * CPS <= 512, "TMEM shared by the CTAs of one SM");
  // Epilogue stage of warp w (4 KB with TMA_OUT, else 2 KB).
  __device__ static constexpr int stage_off(int w) { return kOffStage + w * (kTmaOut ? 4096 : 2048); }
  __device__ static constexpr uint32_t col_s(int b) { return (uint32_t)(b * BN); }
};

__device__ __forceinline__ void store_out(uint4* dst, uint4 v) {
  if (kStreamOut) __stcs(dst, v);
  else *dst = v;
}

// Output gate on 8 bf16 values: bf16(o * bf16(sigmoid(g))), the roundings of the reference's
// separate gate kernel (packed_encoders/_kernels/hybrid.py:196-205).
__device__ __forceinline__ uint4 gate8(uint4 o, uint4 g) {
  const uint32_t ow[4] = {o.x, o.y, o.z, o.w}, gw[4] = {g.x, g.y, g.z, g.w};
  uint32_t y[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float o0 = __uint_as_float(ow[w] << 16), o1 = __uint_as_float(ow[w] & 0xffff0000u);
    const float g0 = __uint_as_float(gw[w] << 16), g1 = __uint_as_float(gw[w] & 0xffff0000u);
    const uint32_t s = pack_bf16x2(__fdividef(1.f, 1.f + __expf(-g0)), __fdividef(1.f, 1.f + __expf(-g1)));
    y[w] = pack_bf16x2(o0 * __uint_as_float(s << 16), o1 * __uint_as_float(s & 0xffff0000u));
  }
  return make_uint4(y[0], y[1], y[2], y[3]);
}

__device__ __forceinline__ uint4 load_gate8(const AttnParams& p, int tok, int head, int col) {
  return __ldg(reinterpret_cast<const uint4*>(p.gate + (long long)tok * p.g_tok + (long long)head * p.g_head + col));
}

// The output gate as its own pass over `out` (in place), for head dims where the fused epilogue
// is slower, with the fused path's roundings (gate8): one 16-byte vector of the
// [token][head][column] output per thread and a grid that covers the tensor (no loop). On config 5
// shapes it runs at 7.1 TB/s (0.94 ms for 6.7 GB, reads twice the writes); two or four vectors
// per thread, streaming cache hints, writing a new tensor and a one-wave persistent grid all
// measured the same or slower.
__global__ void __launch_bounds__(256) gate_pass_kernel(__nv_bfloat16* out, const __nv_bfloat16* gate, int total_q,
                                                        int heads, int vec_per_row, long long o_tok, long long o_head,
                                                        long long g_tok, long long g_head) {
  const long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_tok = heads * vec_per_row;
  if (v >= (long long)total_q * per_tok) return;
  const int t = (int)(v / per_tok);
  const int rem = (int)(v - (long long)t * per_tok);
  const int h = rem / vec_per_row, c = (rem - h * vec_per_row) * 8;
  __nv_bfloat16* op = out + (long long)t * o_tok + (long long)h * o_head + c;
  const uint4 ov = *reinterpret_cast<const uint4*>(op);
  const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gate + (long long)t * g_tok + (long long)h * g_head + c));
  *reinterpret_cast<uint4*>(op) = gate8(ov, gv);
}

// Rotary embedding of q and k (head_dim 64) into contiguous [T, H, 64] / [T, KV, 64] buffers. Work
// item i (grid-stride) = token i / (4 * (H + KV)) and, within it, t = i % (4 * (H + KV)): the 16
// elements of dims {8c..8c+7} and {8c+32..8c+39} (c = t % 4) of one head of q (t < 4H) or k.
// A token's table row is shared by its heads (L1). Per element pair, in fp32 rounded to bf16
// (packed_encoders/_kernels/rope.py:5-6, 140-200; the reference CPU path cpu/attention.py:298-301):
//   y[d] = x[d]*cos[d] - x[d+32]*sin[d],  y[d+32] = x[d+32]*cos[d+32] + x[d]*sin[d+32].
__global__ void __launch_bounds__(256) rope_pass_kernel(const __nv_bfloat16* q, const __nv_bfloat16* k,
                                                        long long q_tok, long long q_head, long long k_tok,
                                                        long long k_head, const __nv_bfloat16* cos_t,
                                                        const __nv_bfloat16* sin_t, long long t_tok, int t_rows,
                                                        int total, int heads, int kv_heads, __nv_bfloat16* q_out,
                                                        __nv_bfloat16* k_out) {
  const int per_tok = 4 * (heads + kv_heads);
  const long long n = (long long)total * per_tok;
  auto e0 = [](uint32_t v) { return __uint_as_float(v << 16); };
  auto e1 = [](uint32_t v) { return __uint_as_float(v & 0xffff0000u); };
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    {
      const int tok = (int)(i / per_tok), t = (int)(i - (long long)tok * per_tok);
      const int c = t & 3, hh = t >> 2;
      const bool is_q = hh < heads;
      const int h = is_q ? hh : hh - heads;
      const __nv_bfloat16* src = is_q ? q + (long long)tok * q_tok + (long long)h * q_head
                                      : k + (long long)tok * k_tok + (long long)h * k_head;
      __nv_bfloat16* dst = is_q ? q_out + ((long long)tok * heads + h) * 64 : k_out + ((long long)tok * kv_heads + h) * 64;
      const int trow = tok < t_rows ? tok : tok % t_rows;  // dense [S, 64] tables over a [B, S] batch
      const uint4* c4 = reinterpret_cast<const uint4*>(cos_t + (long long)trow * t_tok);
      const uint4* s4 = reinterpret_cast<const uint4*>(sin_t + (long long)trow * t_tok);
      const uint4 xl = __ldg(reinterpret_cast<const uint4*>(src) + c), xh = __ldg(reinterpret_cast<const uint4*>(src) + c + 4);
      const uint4 cl = __ldg(c4 + c), ch = __ldg(c4 + c + 4), sl = __ldg(s4 + c), sh = __ldg(s4 + c + 4);
      const uint32_t lo[4] = {xl.x, xl.y, xl.z, xl.w}, hi[4] = {xh.x, xh.y, xh.z, xh.w};
      const uint32_t cl4[4] = {cl.x, cl.y, cl.z, cl.w}, ch4[4] = {ch.x, ch.y, ch.z, ch.w};
      const uint32_t sl4[4] = {sl.x, sl.y, sl.z, sl.w}, sh4[4] = {sh.x, sh.y, sh.z, sh.w};
      uint32_t ylo[4], yhi[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float a0 = e0(lo[w]), a1 = e1(lo[w]), b0 = e0(hi[w]), b1 = e1(hi[w]);
        ylo[w] = pack_bf16x2(a0 * e0(cl4[w]) - b0 * e0(sl4[w]), a1 * e1(cl4[w]) - b1 * e1(sl4[w]));
        yhi[w] = pack_bf16x2(b0 * e0(ch4[w]) + a0 * e0(sh4[w]), b1 * e1(ch4[w]) + a1 * e1(sh4[w]));
      }
      reinterpret_cast<uint4*>(dst)[c] = make_uint4(ylo[0], ylo[1], ylo[2], ylo[3]);
      reinterpret_cast<uint4*>(dst)[c + 4] = make_uint4(yhi[0], yhi[1], yhi[2], yhi[3]);
    }
  }
}

struct UnitInfo {
  int head, kv_head;
  int f, c, qb;
  int q_row0, nq;
  int kv_lo, n_kv;
};

// Segment bounds a unit needs: cu_q[f], cu_q[f + c], cu_k[f], cu_k[f + c] (for one sequence,
// c = 1, the last two are its key segment).
__device__ __forceinline__ int4 unit_bounds(const AttnParams& p, const WorkItem& it) {
  return make_int4(p.cu_q[it.seq_first], p.cu_q[it.seq_first + it.seq_count], p.cu_k[it.seq_first],
                   p.cu_k[it.seq_first + it.seq_count]);
}

// Unit order. Item-major (units u = item * heads + head): the heads of a query block run
// together, so the 256-byte L2 lines of a token's K/V rows (two heads each) are used at once; best
// for windowed layers and batches of short sequences. KV-major (kv_major: KV head, then item, then
// the query heads sharing that KV head): the ~296 units resident at a time cover many query
// blocks of one (sequence, KV head) instead of a few blocks of every head, so the K/V of a long
// sequence is read from DRAM about once and served from L2 to all its query blocks (item-major
// order re-reads it for every wave of resident units the sequence spans).
__device__ __forceinline__ void unit_coords(uint32_t u, uint32_t n_items, uint32_t group, uint32_t heads,
                                            bool kv_major, uint32_t& item, int& head) {
  if (!kv_major) {
    item = u / heads;
    head = (int)(u - item * heads);
    return;
  }
  const uint32_t per_kv = n_items * group;
  const uint32_t kvh = u / per_kv;
  const uint32_t rem = u - kvh * per_kv;
  item = rem / group;
  head = (int)(kvh * group + (rem - item * group));
}

// UnitInfo of a unit from its schedule entry, bounds and head (arithmetic only).
template <int BN>
__device__ __forceinline__ UnitInfo unit_derive(const AttnParams& p, const WorkItem& it, int4 b, int head) {
  UnitInfo ui;
  ui.head = head;
  ui.kv_head = ui.head / p.group;
  ui.f = it.seq_first;
  ui.c = it.seq_count;
  ui.qb = it.q_block;
  ui.q_row0 = b.x + ui.qb * kTileM;
  ui.nq = min(kTileM, b.y - ui.q_row0);
  int kv_lo, kv_hi;
  if (ui.c == 1) {
    int lo, hi;
    block_key_range(ui.qb, ui.nq, b.y - b.x, b.w - b.z, p.window_left, p.window_right, lo, hi);
    kv_lo = b.z + lo;
    kv_hi = b.z + hi;
  } else {
    kv_lo = b.z;
    kv_hi = b.w;
  }
  ui.kv_lo = kv_lo;
  ui.n_kv = (ui.nq > 0 && kv_hi > kv_lo) ? (kv_hi - kv_lo + BN - 1) / BN : 0;
  return ui;
}

// The CTA's units (b, b + grid, ...) for the producer, as a three-stage pipeline so that moving
// to the next unit waits on no global load: the schedule entry of the unit three ahead and the
// segment bounds of the unit two ahead are loaded one advance before they are used, and the next
// unit's UnitInfo is then arithmetic only.
template <int BN>
struct UnitStream {
  uint32_t u, n, step, n_items, group, heads;
  bool kv_major;
  UnitInfo cur, nxt;
  WorkItem it2, it3;  // schedule entries of units u + 2*step, u + 3*step
  int4 b2;            // bounds of unit u + 2*step
  int h2, h3;         // heads of units u + 2*step, u + 3*step
  __device__ __forceinline__ WorkItem item(const AttnParams& p, uint32_t v, int& head) const {
    uint32_t idx;
    unit_coords(v, n_items, group, heads, kv_major, idx, head);
    return p.items[idx];
  }
  __device__ __forceinline__ UnitStream(const AttnParams& p, uint32_t items, uint32_t first, uint32_t stride)
      : u(first), n(items * (uint32_t)p.heads), step(stride), n_items(items), group((uint32_t)p.group),
        heads((uint32_t)p.heads), kv_major(p.kv_major != 0) {
    cur.n_kv = 0;
    nxt.n_kv = 0;
    int h;
    if (u < n) {
      const WorkItem it = item(p, u, h);
      cur = unit_derive<BN>(p, it, unit_bounds(p, it), h);
    }
    if (u + step < n) {
      const WorkItem it = item(p, u + step, h);
      nxt = unit_derive<BN>(p, it, unit_bounds(p, it), h);
    }
    if (u + 2 * step < n) {
      it2 = item(p, u + 2 * step, h2);
      b2 = unit_bounds(p, it2);
    }
    if (u + 3 * step < n) it3 = item(p, u + 3 * step, h3);
  }
  __device__ __forceinline__ bool valid() const { return u < n; }
  __device__ __forceinline__ void advance(const AttnParams& p) {
    u += step;
    cur = nxt;
    if (u + step < n) nxt = unit_derive<BN>(p, it2, b2, h2);
    if (u + 2 * step < n) {
      it2 = it3;
      h2 = h3;
      b2 = unit_bounds(p, it2);
    }
    if (u + 3 * step < n) it3 = item(p, u + 3 * step, h3);
  }
};

// Producer side of the row slot: the unit header and, for each of the 128 rows, the allowed
// key interval [klo, khi) in absolute key tokens (rows past the unit get an empty interval).
// Packed short sequences: the sequence of row tq is f + #(boundaries cu_q[f+1 .. f+c-1] <= tq),
// counted with one coalesced load per 32 boundaries and warp shuffles.
template <class C>
__device__ __forceinline__ void write_row_slot(const AttnParams& p, const UnitInfo& ui, uint8_t* slot_bytes,
                                               int lane) {
  int* hdr = reinterpret_cast<int*>(slot_bytes);
  int2* rows = reinterpret_cast<int2*>(hdr + 16);
  if (lane == 0) {
    hdr[0] = ui.q_row0;
    hdr[1] = ui.nq;
    hdr[2] = ui.head;
    hdr[3] = ui.kv_lo;
    hdr[4] = ui.n_kv;
  }
  int cnt[4] = {0, 0, 0, 0};
  if (ui.c > 1) {
    for (int base = 1; base < ui.c; base += 32) {
      const int idx = base + lane;
      const int v = idx < ui.c ? p.cu_q[ui.f + idx] : 0x7fffffff;
#pragma unroll 4
      for (int j = 0; j < 32; ++j) {
        const int b = __shfl_sync(0xffffffffu, v, j);
#pragma unroll
        for (int g = 0; g < 4; ++g) cnt[g] += (b <= ui.q_row0 + lane + 32 * g) ? 1 : 0;
      }
    }
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int r = lane + 32 * g;
    const int tq = ui.q_row0 + r;
    int klo = 0, khi = 0;
    if (r < ui.nq) {
      const int s = min(ui.f + cnt[g], ui.f + ui.c - 1);
      const int cq = p.cu_q[s], lq = p.cu_q[s + 1] - cq;
      const int ck = p.cu_k[s], lk = p.cu_k[s + 1] - ck;
      const int pos = tq - cq + (lk - lq);
      klo = ck + (p.window_left >= 0 ? max(0, pos - p.window_left) : 0);
      khi = ck + (p.window_right >= 0 ? min(lk, pos + p.window_right + 1) : lk);
    }
    rows[r] = make_int2(klo, khi);
  }
}

// Load `n` consecutive 32-column chunks of this warp's TMEM lanes (no wait).
template <int N>
__device__ __forceinline__ void tmem_ld_chunks(uint32_t taddr, uint32_t (&r)[N * 32]) {
#pragma unroll
  for (int c = 0; c < N; ++c) tmem_ld32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
}

// Non-finite inputs. A key tile's P.V multiplies every key row the tile holds, including rows of
// neighbouring sequences and rows past a segment's end, whose P is 0; 0 x Inf is NaN, so one
// non-finite V row would spread to the other sequences of its tile. The epilogue therefore sums
// a row's O values as they leave TMEM (one NaN or Inf makes the sum non-finite) and rewrites a
// row whose sum is non-finite from its own allowed keys [klo, khi) alone, in fp32 with the tile
// loop's max and sum: a non-finite value then reaches exactly the queries that attend to its key,
// as in a per-sequence computation. Finite inputs never take the rewrite; the check is one
// packed-add tree per row (measured with the packed O / l scaling: +0.6 % on a long-document
// global layer, +1.6 % on a windowed one, +7 % on a batch of very short sequences, where the
// epilogue is a large share of a unit).
__device__ __forceinline__ float2 chunk_sum32(const uint32_t* o, float2 acc) {
  float2 b = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    acc = fadd2(acc, make_float2(__uint_as_float(o[j]), __uint_as_float(o[j + 1])));
    b = fadd2(b, make_float2(__uint_as_float(o[j + 2]), __uint_as_float(o[j + 3])));
  }
  return fadd2(acc, b);
}

// o[0 .. 32) = sum_j exp2(c2 * (q . k_j) - m) * v_j[col0 .. col0 + 32) over keys [klo, khi), in
// fp32 from bf16 rows (qrow: the query row; kbase / vbase: the row of token 0 at the unit's KV
// head). Accumulates in the chunk's own registers.
template <int D>
__device__ __forceinline__ void recompute_chunk(uint32_t* o, const __nv_bfloat16* qrow, const __nv_bfloat16* kbase,
                                                const __nv_bfloat16* vbase, long long k_tok, long long v_tok,
                                                float c2, float m, int klo, int khi, int col0) {
#pragma unroll
  for (int j = 0; j < 32; ++j) o[j] = 0u;
#pragma unroll 1
  for (int key = klo; key < khi; ++key) {
    const uint4* krow = reinterpret_cast<const uint4*>(kbase + (long long)key * k_tok);
    float s = 0.f;
#pragma unroll 1
    for (int d = 0; d < D / 8; ++d) {
      const uint4 a = reinterpret_cast<const uint4*>(qrow)[d];
      const uint4 b = krow[d];
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s = fmaf(__uint_as_float(aw[e] << 16), __uint_as_float(bw[e] << 16), s);
        s = fmaf(__uint_as_float(aw[e] & 0xffff0000u), __uint_as_float(bw[e] & 0xffff0000u), s);
      }
    }
    const float pj = ex2(fmaf(s, c2, -m));
    const uint4* vrow = reinterpret_cast<const uint4*>(vbase + (long long)key * v_tok + col0);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 w = vrow[c];
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        o[c * 8 + 2 * e] = __float_as_uint(fmaf(pj, __uint_as_float(ww[e] << 16), __uint_as_float(o[c * 8 + 2 * e])));
        o[c * 8 + 2 * e + 1] =
            __float_as_uint(fmaf(pj, __uint_as_float(ww[e] & 0xffff0000u), __uint_as_float(o[c * 8 + 2 * e + 1])));
      }
    }
  }
}

template <class C>
__global__ void __launch_bounds__(C::kThreads) __maxnreg__(C::kMaxRegs)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                    const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* k_full = bars;
  uint64_t* k_empty = k_full + C::ST;
  uint64_t* v_full = k_empty + C::ST;
  uint64_t* v_empty = v_full + C::VST;
  uint64_t* q_full = v_empty + C::VST;
  uint64_t* q_empty = q_full + C::QB;
  uint64_t* s_full = q_empty + C::QB;
  uint64_t* p_full = s_full + C::NS;
  uint64_t* o_full = p_full + C::NS;  // the last P.V of each unit (epilogue)
  uint64_t* row_empty = o_full + 1;    // [QB] the softmax warps took the unit's row slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::ST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < C::VST; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < C::QB; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // one arrival per softmax warp
    }
    mbar_init(o_full, 1);
    for (int i = 0; i < C::QB; ++i) mbar_init(&row_empty[i], 4);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t n_items = (uint32_t)p.header->n_items;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // The whole warp runs the loop (uniform control flow); one elected lane issues each copy.
    {
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      auto load_q = [&](void* dst, int c0, int c1, int c2, uint64_t* bar) {
        if (kQEvictFirst) tma_load_3d_hint_w(dst, &tm_q, bar, c0, c1, c2, pol_q);
        else tma_load_3d_w(dst, &tm_q, bar, c0, c1, c2);
      };
      auto load_kv4 = [&](void* dst, const CUtensorMap* map, int row, int kvh, uint64_t* bar) {
        if (kKVPolicy == 1) tma_load_4d_hint_w(dst, map, bar, 0, row, kvh, 0, pol_kv);
        else tma_load_4d_w(dst, map, bar, 0, row, kvh, 0);
      };
      auto load_kv = [&](void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
        if (kKVPolicy == 1) tma_load_3d_hint_w(dst, map, bar, c0, c1, c2, pol_kv);
        else tma_load_3d_w(dst, map, bar, c0, c1, c2);
      };
      // Ring counters are 32-bit unsigned: their division by a stage count (3 for some rings) is a
      // multiply-high, not a 64-bit division, on this warp's issue path.
      uint32_t i = 0;  // key tiles whose K is issued; V of tile i-1 follows K of tile i
      int lu = 0;
      int v_row = 0, v_head = 0;
      bool v_pending = false;
      auto issue_v = [&](uint32_t j, int row, int kvh) {
        const int st = (int)(j % C::VST);
        if (j >= C::VST) mbar_wait(&v_empty[st], (int)((j / C::VST) - 1) & 1, p.err);
        uint8_t* vs = smem + C::kOffV + st * C::kKVBytes;
        mbar_arrive_expect_tx_w(&v_full[st], C::kKVBytes);
        if constexpr (C::kPanels > 1) {
          load_kv4(vs, &tm_v, row, kvh, &v_full[st]);
        } else {
          load_kv(vs, &tm_v, 0, kvh, row, &v_full[st]);
        }
      };
      for (UnitStream<C::BN> us(p, n_items, blockIdx.x, gridDim.x); us.valid(); us.advance(p)) {
        const UnitInfo ui = us.cur;
        if (ui.n_kv == 0) continue;
        const int qb = lu % C::QB;
        if (lu >= C::QB) mbar_wait(&q_empty[qb], ((lu / C::QB) - 1) & 1, p.err);
        // The Q copy goes first (its bytes are expected before the arrival), then the row slot;
        // the producer's arrival on q_full, after the slot stores, publishes both.
        uint8_t* qs = smem + C::kOffQ + qb * C::kQBytes;
        mbar_expect_tx_w(&q_full[qb], C::kQBytes);
        if constexpr (C::kPanels > 1) {
          if (kQEvictFirst) tma_load_4d_hint_w(qs, &tm_q, &q_full[qb], 0, ui.q_row0, ui.head, 0, pol_q);
          else tma_load_4d_w(qs, &tm_q, &q_full[qb], 0, ui.q_row0, ui.head, 0);
        } else {
          load_q(qs, 0, ui.head, ui.q_row0, &q_full[qb]);
        }
        if (lu >= C::QB) mbar_wait(&row_empty[qb], ((lu / C::QB) - 1) & 1, p.err);
        write_row_slot<C>(p, ui, smem + C::kOffRows + qb * C::kRowSlotBytes, lane);
        __syncwarp();  // the slot stores are ordered before the q_full arrival
        if (lane == 0) mbar_arrive(&q_full[qb]);
        for (int t = 0; t < ui.n_kv; ++t, ++i) {
          const int st = (int)(i % C::ST);
          if (i >= C::ST) mbar_wait(&k_empty[st], (int)((i / C::ST) - 1) & 1, p.err);
          const int row = ui.kv_lo + t * C::BN;
          uint8_t* ks = smem + C::kOffK + st * C::kKVBytes;
          mbar_arrive_expect_tx_w(&k_full[st], C::kKVBytes);
          if constexpr (C::kPanels > 1) {
            load_kv4(ks, &tm_k, row, ui.kv_head, &k_full[st]);
          } else {
            load_kv(ks, &tm_k, 0, ui.kv_head, row, &k_full[st]);
          }
          if (v_pending) issue_v(i - 1, v_row, v_head);
          v_pending = true;
          v_row = row;
          v_head = ui.kv_head;
        }
        ++lu;
      }
      if (v_pending) issue_v(i - 1, v_row, v_head);
      {  // end marker for the softmax warps: a slot with n_kv = -1, published through q_full
        const int qb = lu % C::QB;
        if (lu >= C::QB) {
          mbar_wait(&q_empty[qb], ((lu / C::QB) - 1) & 1, p.err);
          mbar_wait(&row_empty[qb], ((lu / C::QB) - 1) & 1, p.err);
        }
        if (lane == 0) reinterpret_cast<int*>(smem + C::kOffRows + qb * C::kRowSlotBytes)[4] = -1;
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full[qb]);
      }
      // Tail: every commit that targets this CTA's barriers has landed before exit.
      for (uint32_t j = (i > C::ST ? i - C::ST : 0); j < i; ++j)
        mbar_wait(&k_empty[j % C::ST], (int)(j / C::ST) & 1, p.err);
      for (uint32_t j = (i > C::VST ? i - C::VST : 0); j < i; ++j)
        mbar_wait(&v_empty[j % C::VST], (int)(j / C::VST) & 1, p.err);
      for (int j = (lu > C::QB ? lu - C::QB : 0); j < lu; ++j) mbar_wait(&q_empty[j % C::QB], (j / C::QB) & 1, p.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (uniform control flow); one elected lane issues each MMA.
    {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(kTileM, C::BN, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(kTileM, C::D, false, true);
      const uint32_t smem_base = smem_u32(smem);
      uint32_t i = 0;
      int lu = 0;
      // P.V runs kLag key tiles behind QK: with a third S buffer the QK two tiles ahead is
      // issued before this tile's P is ready, so S waits one more softmax step less often.
      constexpr int kLag = C::NS >= 3 ? 2 : 1;
      uint32_t pend0 = 0;  // oldest key tile whose P.V is not issued yet (pending tiles are consecutive)
      int npend = 0;
      uint32_t pfirst = 0, plast = 0;  // bit k: pending tile pend0 + k is the first / last of its unit
      auto issue_pv = [&](uint32_t j, int first, int last) {
        const int sb = (int)(j % C::NS);
        const int st = (int)(j % C::VST);
        mbar_wait(&p_full[sb], (int)(j / C::NS) & 1, p.err);
        mbar_wait(&v_full[st], (int)(j / C::VST) & 1, p.err);
        tc_fence_after();
        const uint32_t v_addr = smem_base + C::kOffV + st * C::kKVBytes;
#pragma unroll
        for (int g = 0; g < C::BN / 64; ++g) {  // groups of four 16-key k-steps
          uint64_t bdesc[4];
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) bdesc[k4] = sw128_desc(v_addr + (g * 4 + k4) * 16 * 128, C::kKVPanelBytes, 1024);
          uint32_t a_tm[4];
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) a_tm[k4] = tmem + C::col_s(sb) + (g * 4 + k4) * 8;
          if (g == C::BN / 64 - 1) {
            // The last group carries the commits in the same elected block: one completion per unit
            // (the epilogue waits on it, so it is committed first; with two S buffers the next
            // unit's QK is issued before this P.V, so S-ready no longer implies earlier P.V
            // completions), then the V stage release.
            mma_ts4_commit_w(tmem + C::kColO, a_tm, bdesc, idesc_pv, (g > 0 || !first) ? 1u : 0u, o_full,
                             last ? 1u : 0u, &v_empty[st]);
          } else {
            mma_ts4_w(tmem + C::kColO, a_tm, bdesc, idesc_pv, (g > 0 || !first) ? 1u : 0u);
          }
        }
      };
      auto flush_one = [&]() {
        issue_pv(pend0, (int)(pfirst & 1u), (int)(plast & 1u));
        ++pend0;
        --npend;
        pfirst >>= 1;
        plast >>= 1;
      };
      // Units come from the producer's row slots (published with each Q tile; n_kv < 0 ends the
      // stream), so this warp reads no schedule data from global memory: no load chain sits
      // between a unit's last QK and the P.V flush that its epilogue waits for.
      for (;; ++lu) {
        const int qb = lu % C::QB;
        // The previous unit's last P.Vs go before this unit's first QK: the softmax warps run
        // that unit's epilogue before they can use the new S, so its O is what they wait for.
        while (npend > 0) flush_one();
        mbar_wait(&q_full[qb], (lu / C::QB) & 1, p.err);
        tc_fence_after();
        const int n_kv = reinterpret_cast<const int*>(smem + C::kOffRows + qb * C::kRowSlotBytes)[4];
        if (n_kv < 0) break;
        const uint32_t q_addr = smem_base + C::kOffQ + qb * C::kQBytes;
        if constexpr (C::kQTmem) {
          // Q -> TMEM, 16 columns of the head dim (128 rows x 32 bytes) per copy, read through the
          // same descriptors the SS-form QK would use. Every MMA that read the previous unit's Q
          // has completed: the P.V flush above waited for that unit's last P, which the softmax
          // warps publish only after its S, the last QK's result, was ready. The copies are
          // ordered before the QK MMAs that follow; their commit frees the shared-memory Q.
#pragma unroll
          for (int g = 0; g < C::kPanels; ++g) {
            uint64_t qdesc[4];
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) qdesc[k4] = sw128_desc(q_addr + g * C::kQPanelBytes + k4 * 32, 16, 1024);
            tc_cp4_w(tmem + C::kColQ + g * 32, qdesc);
          }
          mma_commit_w(&q_empty[qb]);
        }
        for (int t = 0; t < n_kv; ++t, ++i) {
          const int st = (int)(i % C::ST);
          const int sb = (int)(i % C::NS);
          // With one S buffer the previous P must be consumed first (issue order = execution order).
          if (C::NS == 1)
            while (npend > 0) flush_one();
          mbar_wait(&k_full[st], (int)(i / C::ST) & 1, p.err);
          tc_fence_after();
          const uint32_t k_addr = smem_base + C::kOffK + st * C::kKVBytes;
#pragma unroll
          for (int g = 0; g < C::D / 64; ++g) {  // one 64-column panel: four 16-deep k-steps
            uint64_t adesc[4], bdesc[4];
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              adesc[k4] = sw128_desc(q_addr + g * C::kQPanelBytes + k4 * 32, 16, 1024);
              bdesc[k4] = sw128_desc(k_addr + g * C::kKVPanelBytes + k4 * 32, 16, 1024);
            }
            if constexpr (C::kQTmem) {
              uint32_t a_tm[4];
#pragma unroll
              for (int k4 = 0; k4 < 4; ++k4) a_tm[k4] = tmem + C::kColQ + (g * 4 + k4) * 8;
              if (g == C::D / 64 - 1)  // S ready, K stage free
                mma_ts4_commit_w(tmem + C::col_s(sb), a_tm, bdesc, idesc_qk, g > 0 ? 1u : 0u, &s_full[sb], 1u,
                                 &k_empty[st]);
              else
                mma_ts4_w(tmem + C::col_s(sb), a_tm, bdesc, idesc_qk, g > 0 ? 1u : 0u);
            } else if (g == C::D / 64 - 1) {  // S ready, K stage free and, after the unit's last tile, Q free
              mma_ss4_commit_w(tmem + C::col_s(sb), adesc, bdesc, idesc_qk, g > 0 ? 1u : 0u, &s_full[sb],
                               &k_empty[st], &q_empty[qb], t == n_kv - 1 ? 1u : 0u);
            } else {
              mma_ss4_w(tmem + C::col_s(sb), adesc, bdesc, idesc_qk, g > 0 ? 1u : 0u);
            }
          }
          if (npend == 0) pend0 = i;
          pfirst |= (t == 0 ? 1u : 0u) << npend;
          plast |= (t == n_kv - 1 ? 1u : 0u) << npend;
          ++npend;
          if (npend > kLag) flush_one();
        }
      }
      while (npend > 0) flush_one();
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    // Warp w (2..5) owns TMEM lane quarter w % 4: query rows 32*(w % 4) .. +31, one per thread.
    constexpr int kCols = C::BN;                // S columns per thread per key tile
    constexpr int kPass = C::kPass;  // S columns held in registers at once
    constexpr int kOCols = C::D;                // O columns per thread
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row of this thread == TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t o_addr = tmem + lane_base + C::kColO;
    const float NEG_INF = -__int_as_float(0x7f800000);
    const float c2 = p.scale_log2;
    uint32_t i = 0;
    // A unit's header and this row's allowed keys [klo, khi) come from the producer's row slot,
    // published with the unit's Q tile (a negative key-tile count ends the stream). The next
    // unit's header is read while this unit's last P.V is still running (before the epilogue's
    // wait for it): neither waits for the other, since the producer publishes a unit's slot
    // without waiting for any epilogue.
    UnitInfo ui;
    int klo = 0, khi = 0;
    auto read_header = [&](int u, UnitInfo& h, int& lo, int& hi) {
      const int qb = u % C::QB;
      mbar_wait(&q_full[qb], (u / C::QB) & 1, p.err);
      const int* slot = reinterpret_cast<const int*>(smem + C::kOffRows + qb * C::kRowSlotBytes);
      h.q_row0 = slot[0];
      h.nq = slot[1];
      h.head = slot[2];
      h.kv_lo = slot[3];
      h.n_kv = slot[4];
      if (h.n_kv < 0) return;
      const int2 kr = reinterpret_cast<const int2*>(slot + 16)[r];
      lo = kr.x;
      hi = kr.y;
      __syncwarp();
      if (lane == 0) mbar_arrive(&row_empty[qb]);
    };
    // Epilogue of unit `eu` (its running max m_e and sum l_e; o_full phase of unit elu): O / l -> bf16
    // rows, LSE in natural log.
    auto epilogue = [&](const UnitInfo& eu, float m_e, float l_e, int elu) {
      const bool row_valid = r < eu.nq;
      const int tq = eu.q_row0 + r;
      const float inv = l_e > 0.f ? 1.f / l_e : 0.f;
      const float2 inv2 = make_float2(inv, inv);  // O / l in packed pairs (same rounding as scalar)
      // Gated calls (rows stored by their own thread): the first gate chunk is in flight while
      // the last P.V completes.
      constexpr int kGateChunk = C::CPS == 1 ? 8 : 4;  // uint4 per 32*kEpi columns
      uint4 g_next[(C::kGate && !C::kStageOut) ? kGateChunk : 1];
      if constexpr (C::kGate && !C::kStageOut) {
        if (row_valid && tq < p.total_q) {
#pragma unroll
          for (int j = 0; j < kGateChunk; ++j) g_next[j] = load_gate8(p, tq, eu.head, j * 8);
        }
      }
      mbar_wait(o_full, elu & 1, p.err);
      tc_fence_after();
      const bool store = row_valid && tq >= 0 && tq < p.total_q;
      // Sum of the row's O values as they leave TMEM: non-finite iff some value is (or the sum of
      // huge finite values overflows, which only costs a recomputation).
      float2 o_sum = make_float2(0.f, 0.f);
      __nv_bfloat16* orow = p.out + (long long)tq * p.o_tok + (long long)eu.head * p.o_head;
      if constexpr (C::kTmaOut) {
        // The warp's 32 rows go to its 4 KB stage, then leave with one TMA store; a previous
        // store from the stage must have finished reading it first.
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
      }
      const bool tma_rows = C::kTmaOut && quarter * 32 + 32 <= eu.nq && eu.q_row0 + quarter * 32 + 32 <= p.total_q;
      if (tma_rows) {
        uint8_t* stage = smem + C::stage_off(quarter);
        uint32_t oo[2][32];  // both 32-column halves of O, one TMEM wait
        tmem_ld32(o_addr, oo[0]);
        tmem_ld32(o_addr + 32, oo[1]);
        tmem_wait_ld();
        o_sum = chunk_sum32(oo[1], chunk_sum32(oo[0], o_sum));
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t* o = oo[hh];
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            {
              const float2 y = fmul2(make_float2(__uint_as_float(o[2 * j]), __uint_as_float(o[2 * j + 1])), inv2);
              pk[j] = pack_bf16x2(y.x, y.y);
            }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 val = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            if constexpr (C::kGate) val = gate8(val, load_gate8(p, tq, eu.head, hh * 32 + c * 8));
            *reinterpret_cast<uint4*>(stage + lane * 128 + (((hh * 4 + c) ^ (lane & 7)) * 16)) = val;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (kStreamOut) tma_store_3d_hint(&tm_o, stage, 0, eu.head, eu.q_row0 + quarter * 32, l2_policy_evict_first());
          else tma_store_3d(&tm_o, stage, 0, eu.head, eu.q_row0 + quarter * 32);
          bulk_commit_group();
        }
      } else if constexpr (C::kStageOut) {
        // 64 output columns per thread, in two 32-column halves: each half of all 32 rows of the
        // warp goes through a 2 KB buffer (16-byte chunk c of row r at r*4 + (c ^ (r/2 % 4)),
        // conflict-free both ways) and leaves as 64-byte row segments, 8 rows per instruction.
        uint4* stage = reinterpret_cast<uint4*>(smem + C::stage_off(quarter));
        uint32_t oo[2][32];  // both 32-column halves of O, one TMEM wait
        tmem_ld32(o_addr, oo[0]);
        tmem_ld32(o_addr + 32, oo[1]);
        tmem_wait_ld();
        o_sum = chunk_sum32(oo[1], chunk_sum32(oo[0], o_sum));
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t* o = oo[hh];
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            {
              const float2 y = fmul2(make_float2(__uint_as_float(o[2 * j]), __uint_as_float(o[2 * j + 1])), inv2);
              pk[j] = pack_bf16x2(y.x, y.y);
            }
#pragma unroll
          for (int c = 0; c < 4; ++c)
            stage[lane * 4 + (c ^ ((lane >> 1) & 3))] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int row = k * 8 + (lane >> 2), c = lane & 3;
            uint4 val = stage[row * 4 + (c ^ ((row >> 1) & 3))];
            const int tr = quarter * 32 + row;  // tile row
            const int tok = eu.q_row0 + tr;
            if (tr < eu.nq && tok < p.total_q) {
              if constexpr (C::kGate) val = gate8(val, load_gate8(p, tok, eu.head, hh * 32 + c * 8));
              store_out(reinterpret_cast<uint4*>(p.out + (long long)tok * p.o_tok + (long long)eu.head * p.o_head +
                                                 hh * 32 + c * 8),
                        val);
            }
          }
          __syncwarp();
        }
      } else {
        constexpr int kEpi = C::CPS == 1 ? 2 : 1;  // 32-column chunks per TMEM load
        // Gated calls: the gate of the next 32*kEpi columns is loaded while this chunk is finished.
        static_assert(!C::kGate || kGateChunk == kEpi * 4, "gate chunk");
#pragma unroll
        for (int cc = 0; cc < kOCols / 32; cc += kEpi) {
          uint32_t o[kEpi * 32];
          tmem_ld_chunks<kEpi>(o_addr + cc * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < kEpi; ++e) o_sum = chunk_sum32(&o[e * 32], o_sum);
          uint32_t pk[kEpi * 16];
#pragma unroll
          for (int j = 0; j < kEpi * 16; ++j)
            {
              const float2 y = fmul2(make_float2(__uint_as_float(o[2 * j]), __uint_as_float(o[2 * j + 1])), inv2);
              pk[j] = pack_bf16x2(y.x, y.y);
            }
          if (store) {
            uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
            uint4 g_cur[C::kGate ? kEpi * 4 : 1];
            if constexpr (C::kGate) {
#pragma unroll
              for (int j = 0; j < kEpi * 4; ++j) g_cur[j] = g_next[j];
              if (cc + kEpi < kOCols / 32) {
#pragma unroll
                for (int j = 0; j < kEpi * 4; ++j)
                  g_next[j] = load_gate8(p, tq, eu.head, (cc + kEpi) * 32 + j * 8);
              }
            }
#pragma unroll
            for (int j = 0; j < kEpi * 4; ++j) {
              uint4 val = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
              if constexpr (C::kGate) val = gate8(val, g_cur[j]);
              store_out(dst + j, val);
            }
          }
        }
      }
      if (store && p.lse != nullptr) {
        const float lse = l_e > 0.f ? (m_e + __log2f(l_e)) * 0.69314718055994531f : NEG_INF;
        p.lse[(long long)eu.head * p.total_q + tq] = lse;
      }
      // Rows with a non-finite output are rewritten from their own keys (recompute_chunk), after
      // the warp's bulk output store has landed.
      const bool nonfinite = store && (__float_as_uint(o_sum.x + o_sum.y) & 0x7f800000u) == 0x7f800000u;
      if (__any_sync(0xffffffffu, nonfinite)) {
        if constexpr (C::kTmaOut) {
          if (lane == 0) {
            bulk_wait_all();
            fence_proxy_async_global();
          }
          __syncwarp();
        }
        if (nonfinite) {
          const int kvh = eu.head / p.group;
          const __nv_bfloat16* qrow = p.q + (long long)tq * p.q_tok + (long long)eu.head * p.q_head;
#pragma unroll 1
          for (int cc = 0; cc < kOCols / 32; ++cc) {
            uint32_t o[32];
            recompute_chunk<C::D>(o, qrow, p.k + (long long)kvh * p.k_head, p.v + (long long)kvh * p.v_head, p.k_tok,
                                  p.v_tok, c2, m_e == NEG_INF ? 0.f : m_e, klo, khi, cc * 32);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 val = make_uint4(pack_bf16x2(__uint_as_float(o[8 * j]) * inv, __uint_as_float(o[8 * j + 1]) * inv),
                                     pack_bf16x2(__uint_as_float(o[8 * j + 2]) * inv, __uint_as_float(o[8 * j + 3]) * inv),
                                     pack_bf16x2(__uint_as_float(o[8 * j + 4]) * inv, __uint_as_float(o[8 * j + 5]) * inv),
                                     pack_bf16x2(__uint_as_float(o[8 * j + 6]) * inv, __uint_as_float(o[8 * j + 7]) * inv));
              if constexpr (C::kGate) val = gate8(val, load_gate8(p, tq, eu.head, cc * 32 + j * 8));
              *reinterpret_cast<uint4*>(orow + cc * 32 + j * 8) = val;
            }
          }
        }
      }
      tc_fence_before();
    };
    read_header(0, ui, klo, khi);
    for (int lu = 0;; ++lu) {
      if (ui.n_kv < 0) break;
      float m_run = NEG_INF, l_run = 0.f;
      for (int t = 0; t < ui.n_kv; ++t, ++i) {
        const int sb = (int)(i % C::NS);
        const uint32_t s_addr = tmem + lane_base + C::col_s(sb);
        const int kt = ui.kv_lo + t * C::BN;
        // Valid columns of my row in this key tile: [c_lo, c_hi).
        const int c_lo = klo - kt, c_hi = khi - kt;
        // Warp-uniform: every lane's row sees all my columns (interior tile), and which of my
        // 32-column chunks hold any allowed key of any lane of this warp.
        // With the whole row in one pass, the S load is issued as soon as S is ready and the
        // warp votes below run while it is in flight.
        constexpr bool kEarlyLd = kCols == kPass;
        uint32_t raw[kPass];
        if (kEarlyLd) {
          mbar_wait(&s_full[sb], (int)(i / C::NS) & 1, p.err);
          tc_fence_after();
#pragma unroll
          for (int cc = 0; cc < kPass / 32; ++cc)
            tmem_ld32(s_addr + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&raw[cc * 32]));
        }
        const bool full = __all_sync(0xffffffffu, c_lo <= 0 && c_hi >= kCols);
        uint32_t active = 0;
#pragma unroll
        for (int cc = 0; cc < kCols / 32; ++cc)
          active |= (__any_sync(0xffffffffu, c_lo < 32 * (cc + 1) && c_hi > 32 * cc && c_lo < c_hi) ? 1u : 0u) << cc;
        if (!kEarlyLd) {
          mbar_wait(&s_full[sb], (int)(i / C::NS) & 1, p.err);
          tc_fence_after();
        }

        // ---- pass 1: row max of the raw scores (scale > 0 commutes with max); four
        // independent chains so the warp does not wait on its own latency.
        float mxs[4] = {NEG_INF, NEG_INF, NEG_INF, NEG_INF};
#pragma unroll
        for (int h = 0; h < kCols / kPass; ++h) {
          if (!kEarlyLd) {
#pragma unroll
            for (int cc = 0; cc < kPass / 32; ++cc)
              if (active & (1u << (h * (kPass / 32) + cc)))
                tmem_ld32(s_addr + h * kPass + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&raw[cc * 32]));
          }
          tmem_wait_ld();
          if (full) {
#pragma unroll
            for (int j = 0; j + 1 < kPass; j += 2)
              mxs[(j >> 1) & 3] = fmax3(mxs[(j >> 1) & 3], __uint_as_float(raw[j]), __uint_as_float(raw[j + 1]));
          } else {
#pragma unroll
            for (int cc = 0; cc < kPass / 32; ++cc) {
              if (!(active & (1u << (h * (kPass / 32) + cc)))) continue;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int col = h * kPass + cc * 32 + j;
                const bool ok = (unsigned)(col - c_lo) < (unsigned)(c_hi - c_lo);
                raw[cc * 32 + j] = ok ? raw[cc * 32 + j] : __float_as_uint(NEG_INF);
                mxs[j & 3] = fmaxf(mxs[j & 3], __uint_as_float(raw[cc * 32 + j]));
              }
            }
          }
        }
        const float mx = fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3]));
        const float m_new = fmaxf(m_run, mx * c2);
        const bool need = (m_run != NEG_INF) && (m_new > m_run + kRescaleThreshold);
        const bool any_need = __any_sync(0xffffffffu, need);
        const float alpha = need ? ex2(m_run - m_new) : 1.f;
        if (m_run == NEG_INF || need) m_run = m_new;
        const float base = (m_run == NEG_INF) ? 0.f : m_run;
        const float2 cc2 = make_float2(c2, c2), nb2 = make_float2(-base, -base);

        // ---- pass 2: p = exp2(s * scale_log2 - m), bf16 pairs written over S, fp32 row sum
        float2 accs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int h = 0; h < kCols / kPass; ++h) {
          if (kCols > kPass) {  // S did not fit in registers: reload this pass's columns
#pragma unroll
            for (int cc = 0; cc < kPass / 32; ++cc)
              if (active & (1u << (h * (kPass / 32) + cc)))
                tmem_ld32(s_addr + h * kPass + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&raw[cc * 32]));
            tmem_wait_ld();
            if (!full) {
#pragma unroll
              for (int cc = 0; cc < kPass / 32; ++cc) {
                if (!(active & (1u << (h * (kPass / 32) + cc)))) continue;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  const int col = h * kPass + cc * 32 + j;
                  const bool ok = (unsigned)(col - c_lo) < (unsigned)(c_hi - c_lo);
                  raw[cc * 32 + j] = ok ? raw[cc * 32 + j] : __float_as_uint(NEG_INF);
                }
              }
            }
          }
#pragma unroll
          for (int cc = 0; cc < kPass / 32; ++cc) {
            uint32_t pk[16];
            if (active & (1u << (h * (kPass / 32) + cc))) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                float2 x = ffma2(make_float2(__uint_as_float(raw[cc * 32 + 2 * j]), __uint_as_float(raw[cc * 32 + 2 * j + 1])),
                                 cc2, nb2);
                float2 e = (j < C::POLY) ? ex2_poly2(x) : make_float2(ex2(x.x), ex2(x.y));
                accs[j & 3] = fadd2(accs[j & 3], e);
                pk[j] = pack_bf16x2(e.x, e.y);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) pk[j] = 0u;
            }
            tmem_st16(s_addr + (h * kPass + cc * 32) / 2, pk);
          }
        }
        // O rescale (rare: the running max grew by more than 2^8) after P is out, so the S
        // registers are free and the previous P.V has had the softmax time to finish.
        if (any_need) {
          // O holds the sum up to the previous key tile: wait for that P.V to land.
          // (v_empty of that tile completes with it; its next phase needs this step's P.)
          mbar_wait(&v_empty[(i - 1) % C::VST], (int)(((i - 1) / C::VST) & 1), p.err);
          tc_fence_after();
#pragma unroll
          for (int cc = 0; cc < kOCols / 32; ++cc) {
            uint32_t o[32];
            tmem_ld32(o_addr + cc * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              float2 v = fmul2(make_float2(__uint_as_float(o[j]), __uint_as_float(o[j + 1])), make_float2(alpha, alpha));
              o[j] = __float_as_uint(v.x);
              o[j + 1] = __float_as_uint(v.y);
            }
            tmem_st32(o_addr + cc * 32, o);
          }
          l_run *= alpha;
        }
        const float2 acc = fadd2(fadd2(accs[0], accs[1]), fadd2(accs[2], accs[3]));
        l_run += acc.x + acc.y;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[sb]);
      }
      UnitInfo next;
      int next_lo = 0, next_hi = 0;
      read_header(lu + 1, next, next_lo, next_hi);
      epilogue(ui, m_run, l_run, lu);
      ui = next;
      klo = next_lo;
      khi = next_hi;
    }
    if (C::kTmaOut && lane == 0) bulk_wait_all();  // output stores complete before the CTA exits
  }

  drain_after_timeout(p.err);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Layout probes: one CTA of 128 threads runs a single QK^T or P.V through the same descriptor
// code as the kernel above.
template <int D>
__global__ void __launch_bounds__(128, 1)
    debug_qk_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k, float* s_out,
                    int* err) {
  constexpr int BN = 128;
  constexpr int kPanels = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ks = smem + kPanels * kTileM * 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ks + kPanels * BN * 128);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bars + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bars[0], kPanels * (kTileM + BN) * 128);
    for (int pn = 0; pn < kPanels; ++pn) {
      tma_load_3d(qs + pn * kTileM * 128, &tm_q, &bars[0], pn * 64, 0, 0);
      tma_load_3d(ks + pn * BN * 128, &tm_k, &bars[0], pn * 64, 0, 0);
    }
    mbar_wait(&bars[0], 0, err);
    tc_fence_after();
    constexpr uint32_t idesc = idesc_bf16_f32(kTileM, BN, false, false);
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t off = (kk & 3) * 32;
      mma_ss(tmem, sw128_desc(smem_u32(qs) + (kk >> 2) * kTileM * 128 + off, 16, 1024),
             sw128_desc(smem_u32(ks) + (kk >> 2) * BN * 128 + off, 16, 1024), idesc, kk > 0);
    }
    mma_commit(&bars[1]);
  }
  __syncwarp();
  mbar_wait(&bars[1], 0, err);
  tc_fence_after();
  const int r = warp * 32 + lane;
  for (int cc = 0; cc < BN / 32; ++cc) {
    uint32_t raw[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + cc * 32, raw);
    tmem_wait_ld();
    for (int j = 0; j < 32; ++j) s_out[r * BN + cc * 32 + j] = __uint_as_float(raw[j]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

template <int D>
__global__ void __launch_bounds__(128, 1)
    debug_pv_kernel(const __grid_constant__ CUtensorMap tm_v, const float* p_in, float* o_out, int* err) {
  constexpr int BN = 128;
  constexpr int kPanels = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* vs = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + kPanels * BN * 128);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bars + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const int r = warp * 32 + lane;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  for (int cc = 0; cc < BN / 32; ++cc) {  // P row r -> bf16 pairs in TMEM columns [0, BN/2)
    uint32_t pk[16];
    for (int j = 0; j < 16; ++j)
      pk[j] = pack_bf16x2(p_in[r * BN + cc * 32 + 2 * j], p_in[r * BN + cc * 32 + 2 * j + 1]);
    tmem_st16(tmem + lane_base + cc * 16, pk);
  }
  tmem_wait_st();
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    tc_fence_after();
    mbar_arrive_expect_tx(&bars[0], kPanels * BN * 128);
    for (int pn = 0; pn < kPanels; ++pn) tma_load_3d(vs + pn * BN * 128, &tm_v, &bars[0], pn * 64, 0, 0);
    mbar_wait(&bars[0], 0, err);
    constexpr uint32_t idesc = idesc_bf16_f32(kTileM, D, false, true);
    for (int kk = 0; kk < BN / 16; ++kk)
      mma_ts(tmem + 256, tmem + kk * 8, sw128_desc(smem_u32(vs) + kk * 16 * 128, BN * 128, 1024), idesc, kk > 0);
    mma_commit(&bars[1]);
  }
  __syncwarp();
  mbar_wait(&bars[1], 0, err);
  tc_fence_after();
  for (int cc = 0; cc < D / 32; ++cc) {
    uint32_t raw[32];
    tmem_ld32(tmem + lane_base + 256 + cc * 32, raw);
    tmem_wait_ld();
    for (int j = 0; j < 32; ++j) o_out[r * D + cc * 32 + j] = __uint_as_float(raw[j]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// [tokens, heads, D] bf16 with element strides (token, head); box = 64 columns x 1 head x rows.
// The CUDA error behind the last PE_B200_ERR_CUDA returned on this host thread.
static thread_local char g_cuda_detail[192] = "";

static int cuda_fail(const char* where, cudaError_t e) {
  snprintf(g_cuda_detail, sizeof(g_cuda_detail), "%s: %s", where, cudaGetErrorString(e));
  return PE_B200_ERR_CUDA;
}

static int launch_status(const char* where) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PE_B200_OK : cuda_fail(where, e);
}

static bool make_map(CUtensorMap* map, const void* base, long long tokens, int heads, int dim, long long tok_stride,
                     long long head_stride, int box_rows,
                     CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)heads, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)head_stride * 2, (cuuint64_t)tok_stride * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Head dims above 64: a 4-D view {64 columns, tokens, heads, D/64 panels} (panel stride 128
// bytes) so one copy brings every 64-column panel of a row block, landing panel-major
// ([panel][row][128 B]) as the MMA descriptors expect.
static bool make_map_panels(CUtensorMap* map, const void* base, long long tokens, int heads, int dim,
                            long long tok_stride, long long head_stride, int box_rows,
                            CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  if (dim <= 64) return make_map(map, base, tokens, heads, dim, tok_stride, head_stride, box_rows, promo);
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {64, (cuuint64_t)tokens, (cuuint64_t)heads, (cuuint64_t)(dim / 64)};
  cuuint64_t strides[3] = {(cuuint64_t)tok_stride * 2, (cuuint64_t)head_stride * 2, 128};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, (cuuint32_t)(dim / 64)};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct DeviceInfo {
  int sms = 0;
  int supported = -1;
};

// Per-device facts, looked up once per device under a lock (calls may come from several host
// threads and devices).
static DeviceInfo& device_info(int dev) {
  static DeviceInfo infos[64];
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  DeviceInfo& d = infos[dev & 63];
  if (d.supported < 0) {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    d.sms = sms;
    d.supported = (major == 10 && minor == 0) ? 1 : 0;
  }
  return d;
}

static int block_n_for(int head_dim) { return head_dim == 256 ? 64 : 128; }

// Output gate: a pass of its own after the attention (default), or fused into the attention
// epilogue (PE_B200_GATE=fused, read once per process). On config 5 shapes (GQA 8/2, causal) the
// pass measured faster at every head dim (64: 3.31 vs 3.43 ms, 128: 4.98 vs 5.10, 256: 7.89 vs
// 8.25): in the fused form the two MUFU operations per element of the sigmoid run on the softmax
// warps between one unit and the next, while the pass streams at memory speed.
static bool gate_as_own_pass() {
  static const bool own_pass = [] {
    const char* e = getenv("PE_B200_GATE");
    return !(e && strcmp(e, "fused") == 0);
  }();
  return own_pass;
}

static long long item_capacity(const PeB200AttnParams* p) {
  return (long long)p->n_seq + (long long)p->total_q / kTileM + 2;
}

// Rotary calls keep their rotated q and k in the workspace, after the schedule (256-byte aligned).
static size_t rope_q_offset(const PeB200AttnParams* p) {
  return ((size_t)kHeaderBytes + sizeof(WorkItem) * (size_t)item_capacity(p) + 255) & ~(size_t)255;
}
static size_t rope_k_offset(const PeB200AttnParams* p) {
  return (rope_q_offset(p) + (size_t)p->total_q * p->heads * p->head_dim * 2 + 255) & ~(size_t)255;
}

static size_t workspace_bytes_for(const PeB200AttnParams* p) {
  if (p->rope_cos) return rope_k_offset(p) + (size_t)p->total_k * p->kv_heads * p->head_dim * 2;
  return (size_t)kHeaderBytes + sizeof(WorkItem) * (size_t)item_capacity(p);
}

enum ValidateLevel { kShapes = 0, kSchedule = 1, kFull = 2 };

static int validate(const PeB200AttnParams* p, int level) {
  if (!p) return PE_B200_ERR_NULL;
  if (p->n_seq < 0 || p->total_q < 0 || p->total_k < 0 || p->heads < 1 || p->kv_heads < 1 ||
      p->heads % p->kv_heads != 0)
    return PE_B200_ERR_SHAPE;
  if (p->head_dim != 64 && p->head_dim != 128 && p->head_dim != 256) return PE_B200_ERR_UNSUPPORTED;
  if (p->window_left < -1 || p->window_right < -1) return PE_B200_ERR_WINDOW;
  if (p->total_q > 0 && p->total_k == 0) return PE_B200_ERR_SHAPE;
  if (level == kShapes) return PE_B200_OK;
  if (!p->cu_seqlens_q || !p->cu_seqlens_k || !p->workspace) return PE_B200_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(p->workspace) & 255) != 0) return PE_B200_ERR_WORKSPACE;
  if (p->workspace_bytes < workspace_bytes_for(p)) return PE_B200_ERR_WORKSPACE;
  if (level == kSchedule) return PE_B200_OK;
  if (p->total_q > 0 && (!p->q || !p->out)) return PE_B200_ERR_NULL;
  if (p->total_k > 0 && (!p->k || !p->v)) return PE_B200_ERR_NULL;
  auto aligned16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->out)) return PE_B200_ERR_STRIDE;
  const int64_t strides[8] = {p->q_stride_token, p->q_stride_head, p->k_stride_token, p->k_stride_head,
                              p->v_stride_token, p->v_stride_head, p->o_stride_token, p->o_stride_head};
  for (int64_t s : strides)
    if (s <= 0 || (s * 2) % 16 != 0) return PE_B200_ERR_STRIDE;
  if (p->gate) {
    if (!aligned16(p->gate)) return PE_B200_ERR_STRIDE;
    if (p->g_stride_token <= 0 || p->g_stride_head <= 0 || (p->g_stride_token * 2) % 16 != 0 ||
        (p->g_stride_head * 2) % 16 != 0)
      return PE_B200_ERR_STRIDE;
  }
  if (p->rope_cos || p->rope_sin) {
    if (!p->rope_cos || !p->rope_sin) return PE_B200_ERR_NULL;
    if (!aligned16(p->rope_cos) || !aligned16(p->rope_sin) || p->rope_stride_token < p->head_dim ||
        (p->rope_stride_token * 2) % 16 != 0)
      return PE_B200_ERR_STRIDE;
    // Tables are per query token and applied to key rows of the same index: self-attention only.
    if (p->head_dim != 64 || p->cu_seqlens_k != p->cu_seqlens_q || p->total_k != p->total_q)
      return PE_B200_ERR_UNSUPPORTED;
  }
  return PE_B200_OK;
}

// KV-major unit order (unit_coords) for unwindowed calls whose longest query segment spans more
// than one wave of resident units (its blocks x heads exceed the grid): then item-major order
// would re-read that sequence's K/V from DRAM for every wave. In that order the K/V maps promote
// L2 fills to 128 bytes (one head's row) instead of 256 (two heads' rows, the second of which
// item-major order uses at once and KV-major order does not). One full-size config 3 global
// launch: DRAM reads 7.39 GB (item-major, 256 B) -> 5.06 GB (KV-major, 256 B) -> 3.65 GB
// (KV-major, 128 B), against 2.77 GB of algorithmic reads.
static bool use_kv_major(const PeB200AttnParams* p, int sms, int cps) {
  const bool windowed = p->window_left >= 0 || (p->window_right >= 0 && !p->causal);
  const long long blocks = ((long long)p->max_seqlen_q + kTileM - 1) / kTileM;
  return !windowed && blocks * p->heads > (long long)sms * cps;
}

template <class C>
static int launch_attention(const PeB200AttnParams* p, cudaStream_t stream, int sms) {
  CUtensorMap tq, tk, tv, to;
  const bool kv_major = use_kv_major(p, sms, C::CPS);
  const CUtensorMapL2promotion kv_promo = kv_major ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B : CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  if (!make_map_panels(&tq, p->q, p->total_q, p->heads, C::D, p->q_stride_token, p->q_stride_head, kTileM) ||
      !make_map_panels(&tk, p->k, p->total_k, p->kv_heads, C::D, p->k_stride_token, p->k_stride_head, C::BN,
                       kv_promo) ||
      !make_map_panels(&tv, p->v, p->total_k, p->kv_heads, C::D, p->v_stride_token, p->v_stride_head, C::BN,
                       kv_promo) ||
      !make_map(&to, p->out, p->total_q, p->heads, C::D, p->o_stride_token, p->o_stride_head, 32))
    return cuda_fail("tensor map encoding", cudaErrorInvalidValue);
  {  // the dynamic shared-memory opt-in, once per (configuration, device), under a lock
    static std::mutex mu;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev & 63]) {
      const cudaError_t e =
          cudaFuncSetAttribute(attn_fwd_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
      if (e != cudaSuccess) return cuda_fail("attn_fwd_kernel shared-memory attribute", e);
      attr_set[dev & 63] = true;
    }
  }
  AttnParams ap;
  ap.cu_q = p->cu_seqlens_q;
  ap.cu_k = p->cu_seqlens_k;
  ap.heads = p->heads;
  ap.group = p->heads / p->kv_heads;
  ap.total_q = p->total_q;
  ap.out = static_cast<__nv_bfloat16*>(p->out);
  ap.o_tok = p->o_stride_token;
  ap.o_head = p->o_stride_head;
  ap.lse = p->lse;
  ap.scale_log2 = p->scale * 1.4426950408889634f;
  ap.window_left = p->window_left;
  ap.window_right = p->causal ? 0 : p->window_right;
  ap.header = static_cast<const WsHeader*>(p->workspace);
  ap.items = reinterpret_cast<const WorkItem*>(static_cast<const uint8_t*>(p->workspace) + kHeaderBytes);
  ap.err = &static_cast<WsHeader*>(p->workspace)->error;
  ap.gate = static_cast<const __nv_bfloat16*>(p->gate);
  ap.g_tok = p->g_stride_token;
  ap.g_head = p->g_stride_head;
  ap.kv_major = kv_major ? 1 : 0;
  ap.q = static_cast<const __nv_bfloat16*>(p->q);
  ap.k = static_cast<const __nv_bfloat16*>(p->k);
  ap.v = static_cast<const __nv_bfloat16*>(p->v);
  ap.q_tok = p->q_stride_token;
  ap.q_head = p->q_stride_head;
  ap.k_tok = p->k_stride_token;
  ap.k_head = p->k_stride_head;
  ap.v_tok = p->v_stride_token;
  ap.v_head = p->v_stride_head;
  const long long units = item_capacity(p) * p->heads;
  const long long slots = (long long)sms * C::CPS;
  const int grid = (int)(units < slots ? units : slots);
  attn_fwd_kernel<C><<<grid, C::kThreads, C::kSmemBytes, stream>>>(tq, tk, tv, to, ap);
  return launch_status("attn_fwd_kernel launch");
}

#include "attn_bwd.cuh"

}  // namespace pe_b200

using namespace pe_b200;

extern "C" {

int pe_b200_abi_version(void) { return PE_B200_ABI_VERSION; }

const char* pe_b200_status_string(int status) {
  switch (status) {
    case PE_B200_OK: return "ok";
    case PE_B200_ERR_NULL: return "a required pointer is NULL";
    case PE_B200_ERR_SHAPE: return "invalid heads / kv_heads / head_dim / token counts";
    case PE_B200_ERR_STRIDE: return "stride or base address not 16-byte aligned (TMA requirement)";
    case PE_B200_ERR_WINDOW: return "window_left / window_right must be >= -1";
    case PE_B200_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case PE_B200_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case PE_B200_ERR_CUDA: return "a CUDA launch or tensor-map call failed";
    case PE_B200_ERR_UNSUPPORTED: return "head_dim must be 64, 128 or 256";
    case PE_B200_ERR_SCRATCH_LIMIT:
      return "call too large for the fixed 1 MiB no-allocation scratch (workspace size > 1 MiB; without rotary "
             "tables: n_seq + total_q/128 + 2 > 65520)";
    default: return "unknown status";
  }
}

const char* pe_b200_last_error_detail(void) { return g_cuda_detail; }

int pe_b200_device_supported(int device) { return device_info(device).supported == 1 ? 1 : 0; }

int pe_b200_attn_workspace_size(const PeB200AttnParams* p, size_t* bytes) {
  int st = validate(p, kShapes);
  if (st != PE_B200_OK) return st;
  if (!bytes) return PE_B200_ERR_NULL;
  *bytes = workspace_bytes_for(p);
  return PE_B200_OK;
}

int pe_b200_build_schedule(const PeB200AttnParams* p, void* stream) {
  int st = validate(p, kSchedule);
  if (st != PE_B200_OK) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PE_B200_ERR_CUDA;
  if (device_info(dev).supported != 1) return PE_B200_ERR_DEVICE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  WsHeader* header = static_cast<WsHeader*>(p->workspace);
  if (p->n_seq == 0 || p->total_q == 0) {
    clear_header_kernel<<<1, 1, 0, s>>>(header);  // an empty schedule
  } else {
    SchedParams sp;
    sp.cu_q = p->cu_seqlens_q;
    sp.cu_k = p->cu_seqlens_k;
    sp.n_seq = p->n_seq;
    sp.total_q = p->total_q;
    sp.total_k = p->total_k;
    sp.window_left = p->window_left;
    sp.window_right = p->causal ? 0 : p->window_right;
    sp.block_n = block_n_for(p->head_dim);
    sp.capacity = (int)item_capacity(p);
    sp.header = header;
    sp.items = reinterpret_cast<WorkItem*>(static_cast<uint8_t*>(p->workspace) + kHeaderBytes);
    schedule_kernel<<<1, kBuilderThreads, 0, s>>>(sp);
  }
  return cudaGetLastError() == cudaSuccess ? PE_B200_OK : PE_B200_ERR_CUDA;
}

int pe_b200_attn_run(const PeB200AttnParams* p, void* stream) {
  int st = validate(p, kFull);
  if (st != PE_B200_OK) return st;
  if (p->n_seq == 0 || p->total_q == 0) return PE_B200_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PE_B200_ERR_CUDA;
  const DeviceInfo& info = device_info(dev);
  if (info.supported != 1) return PE_B200_ERR_DEVICE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->rope_cos) {  // rotary tables (validated: head_dim 64, self-attention): rotate, then attend
    uint8_t* ws = static_cast<uint8_t*>(p->workspace);
    __nv_bfloat16* q_rot = reinterpret_cast<__nv_bfloat16*>(ws + rope_q_offset(p));
    __nv_bfloat16* k_rot = reinterpret_cast<__nv_bfloat16*>(ws + rope_k_offset(p));
    const int grid = (int)(p->total_q < info.sms * 8 ? p->total_q : info.sms * 8);
    rope_pass_kernel<<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(p->q), static_cast<const __nv_bfloat16*>(p->k), p->q_stride_token,
        p->q_stride_head, p->k_stride_token, p->k_stride_head, static_cast<const __nv_bfloat16*>(p->rope_cos),
        static_cast<const __nv_bfloat16*>(p->rope_sin), p->rope_stride_token, p->total_q, p->total_q, p->heads,
        p->kv_heads, q_rot, k_rot);
    st = launch_status("rope_pass_kernel launch");
    if (st != PE_B200_OK) return st;
    PeB200AttnParams r = *p;
    r.rope_cos = r.rope_sin = nullptr;
    r.q = q_rot;
    r.k = k_rot;
    r.q_stride_token = (int64_t)p->heads * 64;
    r.q_stride_head = 64;
    r.k_stride_token = (int64_t)p->kv_heads * 64;
    r.k_stride_head = 64;
    return pe_b200_attn_run(&r, stream);
  }
  if (p->gate && gate_as_own_pass()) {
    PeB200AttnParams ungated = *p;
    ungated.gate = nullptr;
    st = pe_b200_attn_run(&ungated, stream);
    if (st != PE_B200_OK) return st;
    const long long vecs = (long long)p->total_q * p->heads * (p->head_dim / 8);
    if (vecs > 256LL * 0x7fffffffLL) return PE_B200_ERR_SHAPE;
    const int grid = (int)((vecs + 255) / 256);
    gate_pass_kernel<<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(p->out), static_cast<const __nv_bfloat16*>(p->gate),
                                          p->total_q, p->heads, p->head_dim / 8, p->o_stride_token, p->o_stride_head,
                                          p->g_stride_token, p->g_stride_head);
    return launch_status("gate_pass_kernel launch");
  }
  if (p->gate) {  // output gate fused: separate instantiations, so ungated kernels carry no gate code
    switch (p->head_dim) {
      case 64: return launch_attention<Cfg<64, 64, 4, 3, 2, 2, 2, 0, 0, false, true, true, true>>(p, s, info.sms);
      case 128: return launch_attention<Cfg<128, 128, 2, 2, 2, 2, 1, 4, 0, false, true>>(p, s, info.sms);
      case 256: return launch_attention<Cfg<256, 64, 3, 2, 1, 2, 1, 0, 0, false, true, true, true>>(p, s, info.sms);
      default: return PE_B200_ERR_UNSUPPORTED;
    }
  }
  switch (p->head_dim) {
    case 64: {
      const bool windowed = (p->window_left >= 0 || p->window_right >= 0) && !p->causal;
      // 64-key tiles, two CTAs per SM. Windowed layers: three S buffers and the TMA-store
      // epilogue. Batches of short sequences (query batches: units of one or two key tiles) also
      // run P.V two tiles behind QK (config 2 -2.3 %); long global sequences measured +1.4 % so.
      if (windowed) return launch_attention<Cfg<64, 64, 4, 3, 2, 3, 2, 0, 0, true>>(p, s, info.sms);
      if (p->max_seqlen_k > 0 && p->max_seqlen_k <= kTileM)
        return launch_attention<Cfg<64, 64, 4, 3, 2, 3, 2>>(p, s, info.sms);
      return launch_attention<Cfg<64, 64, 4, 3, 2, 2, 2, 0, 0, false, false, true, true>>(p, s, info.sms);
    }
    case 128: return launch_attention<Cfg<128, 128, 2, 2, 2, 2, 1, 4>>(p, s, info.sms);
    case 256: return launch_attention<Cfg<256, 64, 3, 2, 1, 2, 1, 0, 0, false, false, true, true>>(p, s, info.sms);
    default: return PE_B200_ERR_UNSUPPORTED;
  }
}

int pe_b200_attn_fwd(const PeB200AttnParams* p, void* stream) {
  int st = validate(p, kFull);
  if (st != PE_B200_OK) return st;
  st = pe_b200_build_schedule(p, stream);
  if (st != PE_B200_OK) return st;
  return pe_b200_attn_run(p, stream);
}

int pe_b200_attn_bwd_workspace_size(const PeB200AttnBwdParams* p, size_t* bytes) {
  const int st = bwd_validate(p, true);
  if (st != PE_B200_OK) return st;
  if (!bytes) return PE_B200_ERR_NULL;
  *bytes = bwd_workspace_bytes(p);
  return PE_B200_OK;
}

int pe_b200_attn_bwd(const PeB200AttnBwdParams* p, void* stream) {
  int st = bwd_validate(p, false);
  if (st != PE_B200_OK) return st;
  if (p->n_seq == 0 || p->total == 0) return PE_B200_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PE_B200_ERR_CUDA;
  const DeviceInfo& info = device_info(dev);
  if (info.supported != 1) return PE_B200_ERR_DEVICE;
  const PeB200AttnParams sched = bwd_schedule_params(p);
  st = pe_b200_build_schedule(&sched, stream);
  if (st != PE_B200_OK) return st;
  return bwd_run(p, static_cast<cudaStream_t>(stream), info.sms);
}

int pe_b200_rope_qk(const void* q, const void* k, int64_t q_stride_token, int64_t q_stride_head,
                    int64_t k_stride_token, int64_t k_stride_head, const void* cos_table, const void* sin_table,
                    int64_t table_stride_token, int32_t table_rows, int32_t total, int32_t heads, int32_t kv_heads,
                    int32_t head_dim, void* q_out, void* k_out, void* stream) {
  if (total < 0 || heads < 1 || kv_heads < 1 || table_rows < 1) return PE_B200_ERR_SHAPE;
  if (head_dim != 64) return PE_B200_ERR_UNSUPPORTED;
  if (total == 0) return PE_B200_OK;
  if (!q || !k || !cos_table || !sin_table || !q_out || !k_out) return PE_B200_ERR_NULL;
  auto aligned16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (!aligned16(q) || !aligned16(k) || !aligned16(cos_table) || !aligned16(sin_table) || !aligned16(q_out) ||
      !aligned16(k_out))
    return PE_B200_ERR_STRIDE;
  const int64_t strides[5] = {q_stride_token, q_stride_head, k_stride_token, k_stride_head, table_stride_token};
  for (int64_t s : strides)
    if (s <= 0 || (s * 2) % 16 != 0) return PE_B200_ERR_STRIDE;
  if (table_stride_token < 64) return PE_B200_ERR_STRIDE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PE_B200_ERR_CUDA;
  const DeviceInfo& info = device_info(dev);
  if (info.supported != 1) return PE_B200_ERR_DEVICE;
  const long long items = (long long)total * 4 * (heads + kv_heads);
  const long long blocks = (items + 255) / 256;
  const int grid = (int)(blocks < info.sms * 8 ? blocks : info.sms * 8);
  rope_pass_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), q_stride_token, q_stride_head,
      k_stride_token, k_stride_head, static_cast<const __nv_bfloat16*>(cos_table),
      static_cast<const __nv_bfloat16*>(sin_table), table_stride_token, table_rows, total, heads, kv_heads,
      static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_out));
  return launch_status("rope_pass_kernel launch");
}

int pe_b200_debug_qk(const void* q, const void* k, int64_t q_stride_token, int64_t k_stride_token, int rows_q,
                     int rows_k, int head_dim, float* s_out, void* stream) {
  if (!q || !k || !s_out) return PE_B200_ERR_NULL;
  if (rows_q < 1 || rows_k < 1) return PE_B200_ERR_SHAPE;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return PE_B200_ERR_UNSUPPORTED;
  CUtensorMap tq, tk;
  if (!make_map(&tq, q, rows_q, 1, head_dim, q_stride_token, head_dim, kTileM) ||
      !make_map(&tk, k, rows_k, 1, head_dim, k_stride_token, head_dim, 128))
    return PE_B200_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int smem = (head_dim / 64) * (kTileM + 128) * 128 + 64 + 1024;
  int* err = nullptr;
  switch (head_dim) {
#define PE_QK(D)                                                                                         \
  case D:                                                                                                \
    cudaFuncSetAttribute(debug_qk_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);         \
    debug_qk_kernel<D><<<1, 128, smem, s>>>(tq, tk, s_out, err);                                         \
    break;
    PE_QK(64)
    PE_QK(128)
    PE_QK(256)
#undef PE_QK
  }
  return cudaGetLastError() == cudaSuccess ? PE_B200_OK : PE_B200_ERR_CUDA;
}

int pe_b200_debug_pv(const float* p_in, const void* v, int64_t v_stride_token, int rows_k, int head_dim,
                     float* o_out, void* stream) {
  if (!p_in || !v || !o_out) return PE_B200_ERR_NULL;
  if (rows_k < 1) return PE_B200_ERR_SHAPE;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return PE_B200_ERR_UNSUPPORTED;
  CUtensorMap tv;
  if (!make_map(&tv, v, rows_k, 1, head_dim, v_stride_token, head_dim, 128)) return PE_B200_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int smem = (head_dim / 64) * 128 * 128 + 64 + 1024;
  int* err = nullptr;
  switch (head_dim) {
#define PE_PV(D)                                                                                         \
  case D:                                                                                                \
    cudaFuncSetAttribute(debug_pv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);         \
    debug_pv_kernel<D><<<1, 128, smem, s>>>(tv, p_in, o_out, err);                                       \
    break;
    PE_PV(64)
    PE_PV(128)
    PE_PV(256)
#undef PE_PV
  }
  return cudaGetLastError() == cudaSuccess ? PE_B200_OK : PE_B200_ERR_CUDA;
}

}  // extern "C"
