// Packed variable-length attention BACKWARD for B200 (sm_100a): head_dim 64, self-attention
// (one cu_seqlens for queries and keys), any window / causal band, H query heads = KV heads.
// Included into attn_fwd.cu inside namespace pe_b200 (it reuses the forward's tile schedule,
// tensor-map helpers and PTX wrappers).
//
// Given q, k, v, the forward's output o and natural-log LSE, and dO, it computes dq, dk, dv of
//   O = softmax(scale * Q K^T + mask) V  per sequence and head,
// the standard recomputation form (dV = P^T dO; dP = dO V^T; dS = P * (dP - rowsum(dO * O));
// dK = scale * dS^T Q; dQ = scale * dS K with P = exp(scale * S - LSE)).
//
// Work: one UNIT = (a 128-token block of one sequence, or a block-diagonal run of short
// sequences, i.e. one item of the forward's schedule, used here as the KEY block; a head). The
// unit loops over the 128-row query sub-blocks whose rows attend to any of its keys. Per sub-block:
//   S  = Q K^T  and  dP = dO V^T   (tcgen05, M = 128 queries on TMEM lanes, N = 128 keys),
//   P, dS per query row (its LSE and rowsum(dO*O) are one value per thread), written as bf16 to a
//   128B-swizzled [query][key] tile in shared memory, which is both the MN-major A operand of
//   dV += P^T dO and dK += dS^T Q (M = 128 keys) and the K-major A operand of dQ = dS K;
//   dV and dK accumulate in TMEM over the sub-blocks (lanes = keys), dQ goes to TMEM per sub-block
//   and is added into an fp32 accumulator in global memory (vector reductions of whole 128-byte
//   lines, through the sub-block's dS tile, free once dQ is computed), then scaled and converted by
//   a last pass. TMEM: S 128 + dP 128 + dV 64 + dK 64 + dQ 64 = 448 columns (one CTA per SM).
// Overlap: the P and dS tiles are double-buffered, and within a unit the MMA warp issues S and dP
// of the NEXT sub-block before the dV, dK and dQ MMAs of this one, so the compute warps work on the
// next sub-block's P and dS while the tensor core computes this one's gradients.
// Roles (320 threads): warp 0 TMA producer (K, V per unit; Q, dO and a row slot per sub-block),
// warp 1 MMA issuer, warps 2-9 compute: one query row (or, for dK / dV, one key row) per thread and
// half of its columns (warps 2-5 keys 0-63 and dQ columns 0-31 and dV; warps 6-9 keys 64-127, dQ
// columns 32-63 and dK), so two compute warps share each SM sub-partition.

struct BwdParams {
  const int32_t* cu;
  int heads;
  int total;
  int window_left;   // -1 unbounded
  int window_right;  // -1 unbounded; 0 when causal
  float scale_log2;  // scale * log2(e)
  float scale;
  const WsHeader* header;
  const WorkItem* items;
  int* err;
  const float* lse2;  // [H, T] LSE * log2(e)
  const float* dsum;  // [H, T] rowsum(dO * O)
  float* dq_acc;      // [T, H, 64] fp32
  __nv_bfloat16* dk;
  long long dk_tok, dk_head;
  __nv_bfloat16* dv;
  long long dv_tok, dv_head;
};

namespace bwd {
constexpr int kQST = 2;                  // Q / dO ring stages
constexpr int kTile = 128;               // keys per unit, queries per sub-block
constexpr int kTileBytes = kTile * 128;  // 128 rows x 64 bf16
constexpr int kOffK = 0;
constexpr int kOffV = kOffK + kTileBytes;
constexpr int kOffQ = kOffV + kTileBytes;                 // [kQST]
constexpr int kOffDO = kOffQ + kQST * kTileBytes;         // [kQST]
constexpr int kPdsBytes = 2 * kTileBytes;                 // one P or dS tile: 2 panels (keys 0-63, 64-127)
constexpr int kOffP = kOffDO + kQST * kTileBytes;         // [2] P tiles (sub-blocks alternate)
constexpr int kOffDS = kOffP + 2 * kPdsBytes;             // [2] dS tiles
constexpr int kSlotBytes = 64 + kTile * 4;                // header + per query row its key columns (2 x int16)
constexpr int kOffSlot = kOffDS + 2 * kPdsBytes;          // [kQST]
// barriers: kv_full kv_empty qd_full[2] qd_empty[2] row_empty[2] s_full p_ready dq_full dq_free
//           dkv_full dkv_free
constexpr int kNumBars = 2 + 3 * kQST + 6;
constexpr int kOffBar = kOffSlot + kQST * kSlotBytes;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;      // + align slack
constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 320, kColDQ = 384;
constexpr uint32_t kTmemCols = 512;
constexpr int kThreads = 320;
constexpr int kComputeWarps = 8;
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
}  // namespace bwd

// Row slot header fields (ints): the sub-block's first query token, its valid rows, the unit's
// first key token and key count, head, sub-block index in the unit, sub-blocks in the unit
// (negative: end of the stream).
enum { kSlotQt = 0, kSlotNq = 1, kSlotKb = 2, kSlotNk = 3, kSlotHead = 4, kSlotStep = 5, kSlotSteps = 6 };

// D = rowsum(dO * O) and LSE * log2(e) per (token, head) into [H, T], and the fp32 dQ accumulator
// rows zeroed: one thread per (token, head) row.
__global__ void __launch_bounds__(256) bwd_prep_kernel(const __nv_bfloat16* o, long long o_tok, long long o_head,
                                                       const __nv_bfloat16* dout, long long do_tok, long long do_head,
                                                       const float* lse, int total, int heads, float* lse2,
                                                       float* dsum, float* dq_acc) {
  const long long rows = (long long)total * heads;
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(r / heads), h = (int)(r - (long long)t * heads);
    const uint4* op = reinterpret_cast<const uint4*>(o + (long long)t * o_tok + (long long)h * o_head);
    const uint4* dp = reinterpret_cast<const uint4*>(dout + (long long)t * do_tok + (long long)h * do_head);
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 a = __ldg(op + c), b = __ldg(dp + c);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        acc = fmaf(__uint_as_float(aw[w] << 16), __uint_as_float(bw[w] << 16), acc);
        acc = fmaf(__uint_as_float(aw[w] & 0xffff0000u), __uint_as_float(bw[w] & 0xffff0000u), acc);
      }
    }
    dsum[(long long)h * total + t] = acc;
    lse2[(long long)h * total + t] = lse[(long long)h * total + t] * 1.4426950408889634f;
    float4* dq = reinterpret_cast<float4*>(dq_acc + r * 64);
#pragma unroll
    for (int c = 0; c < 16; ++c) dq[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// dq = bf16(scale * dq_acc): one thread per 8 columns of a (token, head) row.
__global__ void __launch_bounds__(256) bwd_dq_kernel(const float* dq_acc, int total, int heads, float scale,
                                                     __nv_bfloat16* dq, long long dq_tok, long long dq_head) {
  const long long n = (long long)total * heads * 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i >> 3;
    const int c = (int)(i & 7);
    const int t = (int)(row / heads), h = (int)(row - (long long)t * heads);
    const float4 a = reinterpret_cast<const float4*>(dq_acc + row * 64)[2 * c];
    const float4 b = reinterpret_cast<const float4*>(dq_acc + row * 64)[2 * c + 1];
    const uint4 y = make_uint4(pack_bf16x2(a.x * scale, a.y * scale), pack_bf16x2(a.z * scale, a.w * scale),
                               pack_bf16x2(b.x * scale, b.y * scale), pack_bf16x2(b.z * scale, b.w * scale));
    reinterpret_cast<uint4*>(dq + (long long)t * dq_tok + (long long)h * dq_head)[c] = y;
  }
}

// The unit's key block and query range. A block of one sequence (count 1): keys = the block's
// tokens, queries = every query that may attend one of them (the band rule read backwards: key
// position j is seen by query positions [j - right, j + left]). A run of short sequences: keys =
// queries = the run's tokens.
struct BwdUnit {
  int kb0, nk;   // first key token, keys
  int q0, q1;    // query token range [q0, q1)
  int f, c;      // first sequence, sequences
  int steps;     // 128-row query sub-blocks
};

__device__ __forceinline__ BwdUnit bwd_unit(const BwdParams& p, const WorkItem& it) {
  BwdUnit u;
  u.f = it.seq_first;
  u.c = it.seq_count;
  const int s0 = p.cu[u.f], send = p.cu[u.f + u.c];
  if (u.c == 1) {
    const int len = send - s0;
    const int j0 = it.q_block * kTileM;
    u.kb0 = s0 + j0;
    u.nk = min(kTileM, len - j0);
    const int lo = p.window_right >= 0 ? max(0, j0 - p.window_right) : 0;
    const int hi = p.window_left >= 0 ? min(len, j0 + u.nk - 1 + p.window_left + 1) : len;
    u.q0 = s0 + lo;
    u.q1 = s0 + max(lo, hi);
  } else {
    u.kb0 = s0;
    u.nk = send - s0;
    u.q0 = s0;
    u.q1 = send;
  }
  u.steps = (u.nk > 0 && u.q1 > u.q0) ? (u.q1 - u.q0 + kTileM - 1) / kTileM : 0;
  return u;
}

// Row slot of one query sub-block: header, and per query row its allowed key columns [lo, hi) of
// the unit's key block (its own sequence intersected with the band; empty past the valid rows).
// Rows of a run of short sequences find their sequence by counting boundaries (one coalesced load
// per 32 boundaries and warp shuffles), as in the forward's row slots.
__device__ __forceinline__ void bwd_write_slot(const BwdParams& p, const BwdUnit& u, int head, int step, int qt,
                                               uint8_t* slot_bytes, int lane) {
  int* hdr = reinterpret_cast<int*>(slot_bytes);
  short2* rows = reinterpret_cast<short2*>(hdr + 16);
  const int nq = min(kTileM, u.q1 - qt);
  if (lane == 0) {
    hdr[kSlotQt] = qt;
    hdr[kSlotNq] = nq;
    hdr[kSlotKb] = u.kb0;
    hdr[kSlotNk] = u.nk;
    hdr[kSlotHead] = head;
    hdr[kSlotStep] = step;
    hdr[kSlotSteps] = u.steps;
  }
  int cnt[4] = {0, 0, 0, 0};
  if (u.c > 1) {
    for (int base = 1; base < u.c; base += 32) {
      const int idx = base + lane;
      const int v = idx < u.c ? p.cu[u.f + idx] : 0x7fffffff;
#pragma unroll 4
      for (int j = 0; j < 32; ++j) {
        const int b = __shfl_sync(0xffffffffu, v, j);
#pragma unroll
        for (int g = 0; g < 4; ++g) cnt[g] += (b <= qt + lane + 32 * g) ? 1 : 0;
      }
    }
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int r = lane + 32 * g;
    int klo = 0, khi = 0;
    if (r < nq) {
      const int s = min(u.f + cnt[g], u.f + u.c - 1);
      const int cs = p.cu[s], len = p.cu[s + 1] - cs;
      const int pos = qt + r - cs;
      klo = cs + (p.window_left >= 0 ? max(0, pos - p.window_left) : 0);
      khi = cs + (p.window_right >= 0 ? min(len, pos + p.window_right + 1) : len);
    }
    // as key columns of the unit's block, clamped to [0, 128] (an empty interval stays empty)
    rows[r] = make_short2((short)min(max(klo - u.kb0, 0), bwd::kTile), (short)min(max(khi - u.kb0, 0), bwd::kTile));
  }
}

__global__ void __launch_bounds__(bwd::kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const BwdParams p) {
  using namespace bwd;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + 1;
  uint64_t* qd_full = bars + 2;              // [kQST]
  uint64_t* qd_empty = qd_full + kQST;       // [kQST]
  uint64_t* row_empty = qd_empty + kQST;     // [kQST]
  uint64_t* s_full = row_empty + kQST;       // S and dP of the sub-block are in TMEM
  uint64_t* p_ready = s_full + 1;            // P and dS are in shared memory (8 warps)
  uint64_t* dq_full = p_ready + 1;           // dQ of the sub-block is in TMEM (all its MMAs done)
  uint64_t* dq_free = dq_full + 1;           // dQ was read out of TMEM (8 warps)
  uint64_t* dkv_full = dq_free + 1;          // the unit's dK and dV are complete
  uint64_t* dkv_free = dkv_full + 1;         // dK and dV were read out of TMEM (8 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int i = 0; i < kQST; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
      mbar_init(&row_empty[i], kComputeWarps);
    }
    mbar_init(s_full, 1);
    mbar_init(p_ready, kComputeWarps);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, kComputeWarps);
    mbar_init(dkv_full, 1);
    mbar_init(dkv_free, kComputeWarps);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    prefetch_tensormap(&tm_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t n_units = (uint32_t)p.header->n_items * (uint32_t)p.heads;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    uint32_t i = 0;  // query sub-blocks issued
    int nu = 0;      // units issued
    for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
      const uint32_t item = u / (uint32_t)p.heads;
      const int head = (int)(u - item * (uint32_t)p.heads);
      const BwdUnit un = bwd_unit(p, p.items[item]);
      if (un.steps == 0) continue;
      if (nu > 0) mbar_wait(kv_empty, (nu - 1) & 1, p.err);
      mbar_arrive_expect_tx_w(kv_full, 2 * kTileBytes);
      tma_load_3d_w(smem + kOffK, &tm_k, kv_full, 0, head, un.kb0);
      tma_load_3d_w(smem + kOffV, &tm_v, kv_full, 0, head, un.kb0);
      ++nu;
      for (int s = 0; s < un.steps; ++s, ++i) {
        const int st = (int)(i % kQST);
        if (i >= kQST) mbar_wait(&qd_empty[st], (int)((i / kQST) - 1) & 1, p.err);
        const int qt = un.q0 + s * kTileM;
        mbar_expect_tx_w(&qd_full[st], 2 * kTileBytes);
        tma_load_3d_w(smem + kOffQ + st * kTileBytes, &tm_q, &qd_full[st], 0, head, qt);
        tma_load_3d_w(smem + kOffDO + st * kTileBytes, &tm_do, &qd_full[st], 0, head, qt);
        if (i >= kQST) mbar_wait(&row_empty[st], (int)((i / kQST) - 1) & 1, p.err);
        bwd_write_slot(p, un, head, s, qt, smem + kOffSlot + st * kSlotBytes, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&qd_full[st]);
      }
    }
    {  // end marker: a slot with a negative step count, published through qd_full
      const int st = (int)(i % kQST);
      if (i >= kQST) {
        mbar_wait(&qd_empty[st], (int)((i / kQST) - 1) & 1, p.err);
        mbar_wait(&row_empty[st], (int)((i / kQST) - 1) & 1, p.err);
      }
      if (lane == 0) reinterpret_cast<int*>(smem + kOffSlot + st * kSlotBytes)[kSlotSteps] = -1;
      __syncwarp();
      if (lane == 0) mbar_arrive(&qd_full[st]);
    }
    // Tail: every commit that targets this CTA's barriers has landed before exit.
    for (uint32_t j = (i > kQST ? i - kQST : 0); j < i; ++j) mbar_wait(&qd_empty[j % kQST], (int)(j / kQST) & 1, p.err);
    if (nu > 0) mbar_wait(kv_empty, (nu - 1) & 1, p.err);
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = idesc_bf16_f32(kTile, kTile, false, false);  // S, dP: M=128 q, N=128 k
    constexpr uint32_t idesc_kv = idesc_bf16_f32(kTile, 64, true, true);     // dV, dK: A, B MN-major
    constexpr uint32_t idesc_q = idesc_bf16_f32(kTile, 64, false, true);     // dQ: A K-major, B MN-major
    const uint32_t sb = smem_u32(smem);
    const uint32_t k_addr = sb + kOffK, v_addr = sb + kOffV;
    int nu = 0;  // units whose K / V were waited for
    int ug = 0;  // units whose gradient MMAs are all issued
    // dV += P^T dO, dK += dS^T Q (A = the [query][key] tile read MN-major: M = keys in two 64-key
    // panels, K = queries in 16-row steps of 2 KB; B = dO / Q read MN-major, N = head dim), then
    // dQ = dS K (A = the dS tile K-major, B = the K tile MN-major) of sub-block j, whose P and dS
    // are in tile buffer j % 2.
    auto issue_grads = [&](uint32_t j, int jst, int jstep, int jsteps) {
      const uint32_t pb = sb + kOffP + (j & 1) * kPdsBytes, db = sb + kOffDS + (j & 1) * kPdsBytes;
      const uint32_t q_addr = sb + kOffQ + jst * kTileBytes, do_addr = sb + kOffDO + jst * kTileBytes;
      if (jstep == 0 && ug > 0) {  // dV / dK accumulate afresh: the previous unit's were read out
        mbar_wait(dkv_free, (ug - 1) & 1, p.err);
        tc_fence_after();
      }
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint64_t a[4], b[4];
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = g * 4 + k4;
          a[k4] = sw128_desc(pb + kk * 2048, kTileBytes, 1024);
          b[k4] = sw128_desc(do_addr + kk * 2048, kTileBytes, 1024);
        }
        mma_ss4_w(tmem + kColDV, a, b, idesc_kv, (jstep > 0 || g > 0) ? 1u : 0u);
      }
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint64_t a[4], b[4];
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = g * 4 + k4;
          a[k4] = sw128_desc(db + kk * 2048, kTileBytes, 1024);
          b[k4] = sw128_desc(q_addr + kk * 2048, kTileBytes, 1024);
        }
        if (g == 1)  // then Q and dO of this sub-block are no longer read
          mma_ss4_commits_w(tmem + kColDK, a, b, idesc_kv, 1u, &qd_empty[jst], &qd_empty[jst], &qd_empty[jst], 1u);
        else
          mma_ss4_w(tmem + kColDK, a, b, idesc_kv, jstep > 0 ? 1u : 0u);
      }
      if (j > 0) mbar_wait(dq_free, (int)((j - 1) & 1), p.err);  // the previous dQ was read out
      tc_fence_after();
      const bool last = jstep == jsteps - 1;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint64_t a[4], b[4];
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = g * 4 + k4;
          a[k4] = sw128_desc(db + g * kTileBytes + k4 * 32, 16, 1024);
          b[k4] = sw128_desc(k_addr + kk * 2048, kTileBytes, 1024);
        }
        if (g == 1)  // dQ ready; after the unit's last sub-block also dK / dV ready and K / V free
          mma_ss4_commits_w(tmem + kColDQ, a, b, idesc_q, 1u, dq_full, dkv_full, kv_empty, last ? 7u : 1u);
        else
          mma_ss4_w(tmem + kColDQ, a, b, idesc_q, 0u);
      }
      if (last) ++ug;
    };
    // The sub-block whose gradient MMAs are not issued yet: within a unit they follow the next
    // sub-block's S and dP. A unit's last sub-block is not held back: its gradients release K and V
    // (kv_empty), which the producer waits for before it loads anything of the next unit, the next
    // sub-block's Q and dO included.
    bool pend = false;
    uint32_t pi = 0;
    int pst = 0, pstep = 0, psteps = 0;
    for (uint32_t i = 0;; ++i) {
      const int st = (int)(i % kQST);
      mbar_wait(&qd_full[st], (int)(i / kQST) & 1, p.err);
      tc_fence_after();
      const int* hdr = reinterpret_cast<const int*>(smem + kOffSlot + st * kSlotBytes);
      const int step = hdr[kSlotStep], steps = hdr[kSlotSteps];
      if (steps < 0) break;
      if (pend) {  // S and dP of the pending sub-block were read out; its P and dS are written
        mbar_wait(p_ready, (int)(pi & 1), p.err);
        tc_fence_after();
      }
      if (step == 0) {  // nothing is pending here: the previous unit's last gradients were issued
        mbar_wait(kv_full, nu & 1, p.err);
        tc_fence_after();
        ++nu;
      }
      const uint32_t q_addr = sb + kOffQ + st * kTileBytes, do_addr = sb + kOffDO + st * kTileBytes;
      {  // S = Q K^T, dP = dO V^T (K-major operands, four 16-deep steps over the head dim)
        uint64_t a[4], b[4];
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          a[k4] = sw128_desc(q_addr + k4 * 32, 16, 1024);
          b[k4] = sw128_desc(k_addr + k4 * 32, 16, 1024);
        }
        mma_ss4_w(tmem + kColS, a, b, idesc_s, 0u);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          a[k4] = sw128_desc(do_addr + k4 * 32, 16, 1024);
          b[k4] = sw128_desc(v_addr + k4 * 32, 16, 1024);
        }
        mma_ss4_commits_w(tmem + kColDP, a, b, idesc_s, 0u, s_full, s_full, s_full, 1u);
      }
      if (pend) issue_grads(pi, pst, pstep, psteps);
      if (step == steps - 1) {  // the unit's last sub-block: its gradients now
        mbar_wait(p_ready, (int)(i & 1), p.err);
        tc_fence_after();
        issue_grads(i, st, step, steps);
        pend = false;
      } else {
        pend = true;
        pi = i;
        pst = st;
        pstep = step;
        psteps = steps;
      }
    }
  } else {
    // ------------------------------------------------------------------ P, dS, dQ, dK, dV rows
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;   // 0: keys 0-63 (panel 0), dQ columns 0-31, dV; 1: keys 64-127, dQ 32-63, dK
    const int r = quarter * 32 + lane;  // TMEM lane: query row (S, dP, dQ) or key row (dK, dV)
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float c2 = p.scale_log2;
    int ug = 0;  // units whose dK / dV were read out
    // dQ of sub-block j out of TMEM and into the fp32 accumulator; after a unit's last sub-block,
    // that unit's dK and dV (TMEM lane r is key row r there) out to dk / dv.
    auto finish = [&](uint32_t j, int qt, int nq, int head, bool last, int kb0, int nk) {
      mbar_wait(dq_full, (int)(j & 1), p.err);
      tc_fence_after();
      uint32_t dq[32];  // my half of the row's 64 dQ columns
      tmem_ld32(tmem + lane_base + kColDQ + half * 32, dq);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      // Add my half-row (32 fp32) into the accumulator with whole 128-byte lines per row: the warp
      // stages its 32 rows in its own rows of sub-block j's dS panel (its dK and dQ MMAs are
      // complete), 128B-swizzled (chunk c of row r at r * 128 + (c ^ r % 8) * 16, so the 32 lanes of
      // a store cover all banks), and reads them back eight lanes per row: each vector reduction
      // then covers four rows' full lines instead of 16 bytes of 32 rows.
      {
        uint8_t* stage = smem + kOffDS + (j & 1) * kPdsBytes + half * kTileBytes;
        uint8_t* row = stage + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) =
              make_uint4(dq[4 * c], dq[4 * c + 1], dq[4 * c + 2], dq[4 * c + 3]);
        __syncwarp();
        const int c = lane & 7;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int rr = quarter * 32 + 4 * k + (lane >> 3);
          const uint4 w = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((c ^ (rr & 7)) << 4));
          if (rr < nq && qt + rr < p.total)
            red_add_v4(p.dq_acc + ((long long)(qt + rr) * p.heads + head) * 64 + half * 32 + 4 * c,
                       __uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z), __uint_as_float(w.w));
        }
        __syncwarp();
      }
      if (!last) return;
      mbar_wait(dkv_full, ug & 1, p.err);
      tc_fence_after();
      uint32_t g[2][32];  // dV (half 0) or dK (half 1) of key row r
      tmem_ld32(tmem + lane_base + (half ? kColDK : kColDV), g[0]);
      tmem_ld32(tmem + lane_base + (half ? kColDK : kColDV) + 32, g[1]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dkv_free);
      ++ug;
      if (r < nk && kb0 + r < p.total) {
        uint4* dst = half ? reinterpret_cast<uint4*>(p.dk + (long long)(kb0 + r) * p.dk_tok + (long long)head * p.dk_head)
                          : reinterpret_cast<uint4*>(p.dv + (long long)(kb0 + r) * p.dv_tok + (long long)head * p.dv_head);
        const float sc = half ? p.scale : 1.f;  // dK = scale * dS^T Q
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          const uint32_t* v = &g[c8 >> 2][(c8 & 3) * 8];
          dst[c8] = make_uint4(pack_bf16x2(__uint_as_float(v[0]) * sc, __uint_as_float(v[1]) * sc),
                               pack_bf16x2(__uint_as_float(v[2]) * sc, __uint_as_float(v[3]) * sc),
                               pack_bf16x2(__uint_as_float(v[4]) * sc, __uint_as_float(v[5]) * sc),
                               pack_bf16x2(__uint_as_float(v[6]) * sc, __uint_as_float(v[7]) * sc));
        }
      }
    };
    // The previous sub-block, whose dQ (and dK / dV) are read out after this one's P and dS are
    // written: its gradient MMAs run on the tensor core meanwhile.
    bool pend = false;
    uint32_t pi = 0;
    int pqt = 0, pnq = 0, phead = 0, pkb0 = 0, pnk = 0;
    bool plast = false;
    // Within a unit the next sub-block starts 128 query rows further on: its rows' LSE and
    // rowsum(dO * O) are loaded while this sub-block's dQ is read out.
    bool have_next = false;
    float next_lse2 = 0.f, next_dsum = 0.f;
    for (uint32_t i = 0;; ++i) {
      const int st = (int)(i % kQST);
      mbar_wait(&qd_full[st], (int)(i / kQST) & 1, p.err);
      const int* hdr = reinterpret_cast<const int*>(smem + kOffSlot + st * kSlotBytes);
      const int qt = hdr[kSlotQt], nq = hdr[kSlotNq], kb0 = hdr[kSlotKb], nk = hdr[kSlotNk];
      const int head = hdr[kSlotHead], step = hdr[kSlotStep], steps = hdr[kSlotSteps];
      if (steps < 0) break;
      const short2 kr = reinterpret_cast<const short2*>(hdr + 16)[r];
      __syncwarp();
      if (lane == 0) mbar_arrive(&row_empty[st]);
      const bool row_valid = r < nq;
      const long long hrow = (long long)head * p.total + qt + r;
      const float lse2 = row_valid ? (have_next ? next_lse2 : p.lse2[hrow]) : 0.f;
      const float dsum = row_valid ? (have_next ? next_dsum : p.dsum[hrow]) : 0.f;
      const int c_lo = kr.x, c_hi = kr.y;  // my allowed key columns
      // This tile buffer was last read by the gradient MMAs of sub-block i - 2, complete since
      // finish(i - 2) waited for their dQ.
      uint8_t* p_row = smem + kOffP + (i & 1) * kPdsBytes + r * 128;
      uint8_t* ds_row = smem + kOffDS + (i & 1) * kPdsBytes + r * 128;
      mbar_wait(s_full, (int)(i & 1), p.err);
      tc_fence_after();
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {  // my 64 keys, 32 at a time
        const int cc = 2 * half + h2;   // 32-key chunk of the 128 keys
        uint32_t s[32], dp[32];
        tmem_ld32(tmem + lane_base + kColS + cc * 32, s);
        tmem_ld32(tmem + lane_base + kColDP + cc * 32, dp);
        tmem_wait_ld();
        uint32_t pk[16], dk16[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int col0 = cc * 32 + 2 * j;
          const bool ok0 = (unsigned)(col0 - c_lo) < (unsigned)(c_hi - c_lo);
          const bool ok1 = (unsigned)(col0 + 1 - c_lo) < (unsigned)(c_hi - c_lo);
          // packed f32x2 arithmetic: the same roundings as the scalar form, half the instructions
          const float2 x = ffma2(make_float2(__uint_as_float(s[2 * j]), __uint_as_float(s[2 * j + 1])),
                                 make_float2(c2, c2), make_float2(-lse2, -lse2));
          const float p0 = ok0 ? ex2(x.x) : 0.f;
          const float p1 = ok1 ? ex2(x.y) : 0.f;
          pk[j] = pack_bf16x2(p0, p1);
          const float2 d = fadd2(make_float2(__uint_as_float(dp[2 * j]), __uint_as_float(dp[2 * j + 1])),
                                 make_float2(-dsum, -dsum));
          const float2 g = fmul2(make_float2(p0, p1), d);
          dk16[j] = pack_bf16x2(g.x, g.y);
        }
        // chunks 4*h2 .. +3 of panel `half`, swizzled by the row
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int ch = (h2 * 4 + q4) ^ (r & 7);
          *reinterpret_cast<uint4*>(p_row + half * kTileBytes + (ch << 4)) =
              make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
          *reinterpret_cast<uint4*>(ds_row + half * kTileBytes + (ch << 4)) =
              make_uint4(dk16[4 * q4], dk16[4 * q4 + 1], dk16[4 * q4 + 2], dk16[4 * q4 + 3]);
        }
      }
      fence_proxy_async_smem();  // P and dS visible to the tensor core
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      have_next = step < steps - 1;
      if (have_next) {
        const bool ok = qt + kTileM + r < p.total;
        next_lse2 = ok ? p.lse2[hrow + kTileM] : 0.f;
        next_dsum = ok ? p.dsum[hrow + kTileM] : 0.f;
      }
      if (pend) finish(pi, pqt, pnq, phead, plast, pkb0, pnk);
      pend = true;
      pi = i;
      pqt = qt;
      pnq = nq;
      phead = head;
      plast = step == steps - 1;
      pkb0 = kb0;
      pnk = nk;
    }
    if (pend) finish(pi, pqt, pnq, phead, plast, pkb0, pnk);
  }

  drain_after_timeout(p.err);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side of the backward.
static PeB200AttnParams bwd_schedule_params(const PeB200AttnBwdParams* p) {
  PeB200AttnParams s = {};
  s.cu_seqlens_q = s.cu_seqlens_k = p->cu_seqlens;
  s.n_seq = p->n_seq;
  s.total_q = s.total_k = p->total;
  s.max_seqlen_q = s.max_seqlen_k = p->max_seqlen;
  s.heads = s.kv_heads = 1;
  s.head_dim = 64;
  s.window_left = p->window_left;
  s.window_right = p->window_right;
  s.causal = p->causal;
  s.scale = 1.f;
  s.q_stride_token = s.q_stride_head = s.k_stride_token = s.k_stride_head = 8;
  s.v_stride_token = s.v_stride_head = s.o_stride_token = s.o_stride_head = 8;
  s.workspace = p->workspace;
  s.workspace_bytes = p->workspace_bytes;
  return s;
}

// Workspace: [schedule (header + items)] [dq accumulator fp32 T x H x 64] [lse2 H x T] [dsum H x T],
// each part 256-byte aligned.
static size_t bwd_off_dq(const PeB200AttnBwdParams* p) {
  const PeB200AttnParams s = bwd_schedule_params(p);
  return (workspace_bytes_for(&s) + 255) & ~(size_t)255;
}
static size_t bwd_off_lse2(const PeB200AttnBwdParams* p) {
  return (bwd_off_dq(p) + (size_t)p->total * p->heads * 64 * 4 + 255) & ~(size_t)255;
}
static size_t bwd_off_dsum(const PeB200AttnBwdParams* p) {
  return (bwd_off_lse2(p) + (size_t)p->total * p->heads * 4 + 255) & ~(size_t)255;
}
static size_t bwd_workspace_bytes(const PeB200AttnBwdParams* p) {
  return bwd_off_dsum(p) + (size_t)p->total * p->heads * 4;
}

static int bwd_validate(const PeB200AttnBwdParams* p, bool shapes_only) {
  if (!p) return PE_B200_ERR_NULL;
  if (p->n_seq < 0 || p->total < 0 || p->heads < 1 || p->max_seqlen < 0) return PE_B200_ERR_SHAPE;
  if (p->head_dim != 64) return PE_B200_ERR_UNSUPPORTED;
  if (p->window_left < -1 || p->window_right < -1) return PE_B200_ERR_WINDOW;
  if (shapes_only) return PE_B200_OK;
  if (!p->cu_seqlens || !p->workspace) return PE_B200_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(p->workspace) & 255) != 0 || p->workspace_bytes < bwd_workspace_bytes(p))
    return PE_B200_ERR_WORKSPACE;
  if (p->total == 0 || p->n_seq == 0) return PE_B200_OK;
  const void* ptrs[9] = {p->q, p->k, p->v, p->out, p->dout, p->dq, p->dk, p->dv, p->lse};
  for (const void* ptr : ptrs)
    if (!ptr) return PE_B200_ERR_NULL;
  for (const void* ptr : ptrs)
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return PE_B200_ERR_STRIDE;
  const int64_t strides[16] = {p->q_stride_token,  p->q_stride_head,  p->k_stride_token,  p->k_stride_head,
                               p->v_stride_token,  p->v_stride_head,  p->o_stride_token,  p->o_stride_head,
                               p->do_stride_token, p->do_stride_head, p->dq_stride_token, p->dq_stride_head,
                               p->dk_stride_token, p->dk_stride_head, p->dv_stride_token, p->dv_stride_head};
  for (int64_t s : strides)
    if (s <= 0 || (s * 2) % 16 != 0) return PE_B200_ERR_STRIDE;
  return PE_B200_OK;
}

static int bwd_run(const PeB200AttnBwdParams* p, cudaStream_t s, int sms) {
  uint8_t* ws = static_cast<uint8_t*>(p->workspace);
  float* dq_acc = reinterpret_cast<float*>(ws + bwd_off_dq(p));
  float* lse2 = reinterpret_cast<float*>(ws + bwd_off_lse2(p));
  float* dsum = reinterpret_cast<float*>(ws + bwd_off_dsum(p));
  const long long rows = (long long)p->total * p->heads;
  const int prep_grid = (int)((rows + 255) / 256 < (long long)sms * 8 ? (rows + 255) / 256 : (long long)sms * 8);
  bwd_prep_kernel<<<prep_grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(p->out), p->o_stride_token,
                                            p->o_stride_head, static_cast<const __nv_bfloat16*>(p->dout),
                                            p->do_stride_token, p->do_stride_head, p->lse, p->total, p->heads, lse2,
                                            dsum, dq_acc);
  int st = launch_status("bwd_prep_kernel launch");
  if (st != PE_B200_OK) return st;
  CUtensorMap tq, tk, tv, tdo;
  if (!make_map(&tq, p->q, p->total, p->heads, 64, p->q_stride_token, p->q_stride_head, bwd::kTile) ||
      !make_map(&tk, p->k, p->total, p->heads, 64, p->k_stride_token, p->k_stride_head, bwd::kTile) ||
      !make_map(&tv, p->v, p->total, p->heads, 64, p->v_stride_token, p->v_stride_head, bwd::kTile) ||
      !make_map(&tdo, p->dout, p->total, p->heads, 64, p->do_stride_token, p->do_stride_head, bwd::kTile))
    return cuda_fail("tensor map encoding", cudaErrorInvalidValue);
  {
    static std::mutex mu;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev & 63]) {
      const cudaError_t e = cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 bwd::kSmemBytes);
      if (e != cudaSuccess) return cuda_fail("attn_bwd_kernel shared-memory attribute", e);
      attr_set[dev & 63] = true;
    }
  }
  BwdParams bp;
  bp.cu = p->cu_seqlens;
  bp.heads = p->heads;
  bp.total = p->total;
  bp.window_left = p->window_left;
  bp.window_right = p->causal ? 0 : p->window_right;
  bp.scale_log2 = p->scale * 1.4426950408889634f;
  bp.scale = p->scale;
  bp.header = static_cast<const WsHeader*>(p->workspace);
  bp.items = reinterpret_cast<const WorkItem*>(ws + kHeaderBytes);
  bp.err = &static_cast<WsHeader*>(p->workspace)->error;
  bp.lse2 = lse2;
  bp.dsum = dsum;
  bp.dq_acc = dq_acc;
  bp.dk = static_cast<__nv_bfloat16*>(p->dk);
  bp.dk_tok = p->dk_stride_token;
  bp.dk_head = p->dk_stride_head;
  bp.dv = static_cast<__nv_bfloat16*>(p->dv);
  bp.dv_tok = p->dv_stride_token;
  bp.dv_head = p->dv_stride_head;
  const PeB200AttnParams sched = bwd_schedule_params(p);
  const long long units = item_capacity(&sched) * p->heads;
  const int grid = (int)(units < sms ? units : sms);
  attn_bwd_kernel<<<grid, bwd::kThreads, bwd::kSmemBytes, s>>>(tq, tk, tv, tdo, bp);
  st = launch_status("attn_bwd_kernel launch");
  if (st != PE_B200_OK) return st;
  const long long n = rows * 8;
  const int dq_grid = (int)((n + 255) / 256 < (long long)sms * 8 ? (n + 255) / 256 : (long long)sms * 8);
  bwd_dq_kernel<<<dq_grid, 256, 0, s>>>(dq_acc, p->total, p->heads, p->scale, static_cast<__nv_bfloat16*>(p->dq),
                                        p->dq_stride_token, p->dq_stride_head);
  return launch_status("bwd_dq_kernel launch");
}
