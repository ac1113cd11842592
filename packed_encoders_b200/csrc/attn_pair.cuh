// Two query tiles per CTA (head_dim 64), one CTA per SM.
//
// A pair unit is (work items 2p and 2p+1 of the schedule, one head): tile A and tile B, 128
// query rows each. When both tiles are query blocks of one long sequence whose key ranges sit
// on the same BN-row grid (global and causal layers; local layers past the first block), one
// K/V stream serves both: each key tile is loaded once and used by every tile whose range
// contains it. Otherwise (packed short sequences, different sequences) the two key-tile lists
// are interleaved A0, B0, A1, B1, ... so both tiles still progress together.
//
// Warps: 0 TMA producer, 1 MMA issuer (2-3 idle), 4-7 softmax of tile A, 8-11 softmax of tile B
// (each group covers the four 32-lane TMEM quarters). TMEM: S_A, S_B (BN fp32 columns each, bf16 P
// written over the first BN/2), O_A, O_B (64 columns each). One S buffer per tile: QK of tile
// X's next key tile is issued after its P.V, and the other tile's softmax runs meanwhile, so
// the two softmax groups alternate on the MUFU units of each SM sub-partition.
//
// With one S buffer per tile, the commit that publishes S_X(j) also covers P.V_X(j-1) (a
// tcgen05.commit tracks every earlier MMA of the issuing thread), so the softmax may rescale O_X
// as soon as it sees S_X(j).

template <int BN_, int ST_, int VST_, int QB_, int PASS_ = 64>
struct PairCfg {
  static constexpr int D = 64;
  static constexpr int BN = BN_, ST = ST_, VST = VST_, QB = QB_;
  static constexpr int kThreads = 384;  // three warpgroups at 168 registers per thread
  static constexpr int kPass = PASS_;
  static constexpr int kQBytes = kTileM * 128;  // one 64-column panel of 128 rows
  static constexpr int kKVBytes = BN * 128;
  static constexpr int kOffQ = 0;  // [tile][QB]
  static constexpr int kOffK = kOffQ + 2 * QB * kQBytes;
  static constexpr int kOffV = kOffK + ST * kKVBytes;
  static constexpr int kOffStage = kOffV + VST * kKVBytes;  // 8 softmax warps x 2 KB
  static constexpr int kOffBar = kOffStage + 8 * 2048;
  // k_full[ST] k_empty[ST] v_full[VST] v_empty[VST] q_full[2][QB] q_empty[2][QB] s_full[2] p_full[2] o_full[2]
  static constexpr int kNumBars = 2 * ST + 2 * VST + 4 * QB + 6;
  static constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + align slack
  static constexpr uint32_t kTmemCols = 512;
  __device__ static constexpr uint32_t col_s(int x) { return (uint32_t)(x * BN); }
  __device__ static constexpr uint32_t col_o(int x) { return (uint32_t)(2 * BN + x * 64); }
  static_assert(2 * BN + 128 <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static_assert(BN % 32 == 0 && BN <= 128, "key tile");
};

struct PairInfo {
  UnitInfo t[2];  // t[1].n_kv == 0 when the pair has no second tile
  int shared;     // 1: one key-tile stream for both tiles
  int lo;         // shared: first key row of the stream
  int n;          // key tiles in the stream
};

template <int BN>
__device__ __forceinline__ PairInfo pair_info(const AttnParams& p, long long pp, int n_items) {
  PairInfo pi;
  const long long head = pp % p.heads;
  const long long ia = 2 * (pp / p.heads);
  pi.t[0] = unit_info<BN>(p, ia * p.heads + head);
  pi.t[1].n_kv = 0;
  pi.t[1].nq = 0;
  if (ia + 1 < n_items) pi.t[1] = unit_info<BN>(p, (ia + 1) * p.heads + head);
  const UnitInfo& a = pi.t[0];
  const UnitInfo& b = pi.t[1];
  const int end_a = a.kv_lo + a.n_kv * BN, end_b = b.kv_lo + b.n_kv * BN;
  pi.shared = a.n_kv > 0 && b.n_kv > 0 && a.c == 1 && b.c == 1 && a.f == b.f && ((b.kv_lo - a.kv_lo) % BN) == 0 &&
              max(a.kv_lo, b.kv_lo) <= min(end_a, end_b);
  if (pi.shared) {
    pi.lo = min(a.kv_lo, b.kv_lo);
    pi.n = (max(end_a, end_b) - pi.lo) / BN;
  } else {
    pi.lo = 0;
    pi.n = a.n_kv + b.n_kv;
  }
  return pi;
}

// Key tile t of a pair's stream: its first key row and which tiles use it (bit 0 A, bit 1 B).
template <int BN>
__device__ __forceinline__ void stream_tile(const PairInfo& pi, int t, int& row, int& mask) {
  if (pi.shared) {
    row = pi.lo + t * BN;
    mask = 0;
#pragma unroll
    for (int x = 0; x < 2; ++x)
      if (row >= pi.t[x].kv_lo && row < pi.t[x].kv_lo + pi.t[x].n_kv * BN) mask |= 1 << x;
  } else {
    const int m = min(pi.t[0].n_kv, pi.t[1].n_kv);
    int x, j;
    if (t < 2 * m) {
      x = t & 1;
      j = t >> 1;
    } else {
      x = pi.t[0].n_kv > pi.t[1].n_kv ? 0 : 1;
      j = m + (t - 2 * m);
    }
    row = pi.t[x].kv_lo + j * BN;
    mask = 1 << x;
  }
}

// The CTA's pair units with the next one's info loaded one unit ahead.
template <int BN>
struct PairStream {
  long long u, n, step;
  int n_items;
  PairInfo cur, nxt;
  __device__ __forceinline__ PairStream(const AttnParams& p, long long first, long long n_pairs, long long stride,
                                        int items)
      : u(first), n(n_pairs), step(stride), n_items(items) {
    cur.n = 0;
    nxt.n = 0;
    if (u < n) cur = pair_info<BN>(p, u, n_items);
    if (u + step < n) nxt = pair_info<BN>(p, u + step, n_items);
  }
  __device__ __forceinline__ bool valid() const { return u < n; }
  __device__ __forceinline__ void advance(const AttnParams& p) {
    u += step;
    cur = nxt;
    if (u + step < n) nxt = pair_info<BN>(p, u + step, n_items);
  }
};

// 384 threads = three warpgroups (control, softmax A, softmax B) at 168 registers per thread.
template <class C>
__global__ void __launch_bounds__(C::kThreads, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* k_full = bars;
  uint64_t* k_empty = k_full + C::ST;
  uint64_t* v_full = k_empty + C::ST;
  uint64_t* v_empty = v_full + C::VST;
  uint64_t* q_full = v_empty + C::VST;  // [2][QB]
  uint64_t* q_empty = q_full + 2 * C::QB;
  uint64_t* s_full = q_empty + 2 * C::QB;  // [2]
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
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
    for (int i = 0; i < 2 * C::QB; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);  // one arrival per softmax warp of the tile
      mbar_init(&o_full[x], 1);
    }
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
  const int n_items = p.header->n_items;
  const long long n_pairs = (long long)((n_items + 1) / 2) * p.heads;

  if (warp < 4) {
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    const uint64_t pol_q = l2_policy_evict_first();
    long long i = 0;  // key tiles issued (K of tile i is issued before V of tile i-1)
    int ux[2] = {0, 0};
    int v_row = 0, v_head = 0;
    bool v_pending = false;
    auto issue_v = [&](long long j, int row, int kvh) {
      const int st = (int)(j % C::VST);
      if (j >= C::VST) mbar_wait(&v_empty[st], (int)((j / C::VST) - 1) & 1, p.err);
      mbar_arrive_expect_tx_w(&v_full[st], C::kKVBytes);
      tma_load_3d_w(smem + C::kOffV + st * C::kKVBytes, &tm_v, &v_full[st], 0, kvh, row);
    };
    for (PairStream<C::BN> ps(p, blockIdx.x, n_pairs, gridDim.x, n_items); ps.valid(); ps.advance(p)) {
      const PairInfo& pi = ps.cur;
      if (pi.n == 0) continue;
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (pi.t[x].n_kv == 0) continue;
        const int qb = ux[x] % C::QB;
        uint64_t* qf = &q_full[x * C::QB + qb];
        if (ux[x] >= C::QB) mbar_wait(&q_empty[x * C::QB + qb], ((ux[x] / C::QB) - 1) & 1, p.err);
        mbar_arrive_expect_tx_w(qf, C::kQBytes);
        tma_load_3d_hint_w(smem + C::kOffQ + (x * C::QB + qb) * C::kQBytes, &tm_q, qf, 0, pi.t[x].head,
                           pi.t[x].q_row0, pol_q);
      }
      const int kvh = pi.t[0].n_kv > 0 ? pi.t[0].kv_head : pi.t[1].kv_head;
      for (int t = 0; t < pi.n; ++t, ++i) {
        int row, mask;
        stream_tile<C::BN>(pi, t, row, mask);
        const int st = (int)(i % C::ST);
        if (i >= C::ST) mbar_wait(&k_empty[st], (int)((i / C::ST) - 1) & 1, p.err);
        mbar_arrive_expect_tx_w(&k_full[st], C::kKVBytes);
        tma_load_3d_w(smem + C::kOffK + st * C::kKVBytes, &tm_k, &k_full[st], 0, kvh, row);
        if (v_pending) issue_v(i - 1, v_row, v_head);
        v_pending = true;
        v_row = row;
        v_head = kvh;
      }
#pragma unroll
      for (int x = 0; x < 2; ++x)
        if (pi.t[x].n_kv > 0) ++ux[x];
    }
    if (v_pending) issue_v(i - 1, v_row, v_head);
    // Tail: every commit that targets this CTA's barriers has landed before exit.
    for (long long j = (i > C::ST ? i - C::ST : 0); j < i; ++j)
      mbar_wait(&k_empty[j % C::ST], (int)(j / C::ST) & 1, p.err);
    for (long long j = (i > C::VST ? i - C::VST : 0); j < i; ++j)
      mbar_wait(&v_empty[j % C::VST], (int)(j / C::VST) & 1, p.err);
#pragma unroll
    for (int x = 0; x < 2; ++x)
      for (int j = (ux[x] > C::QB ? ux[x] - C::QB : 0); j < ux[x]; ++j)
        mbar_wait(&q_empty[x * C::QB + j % C::QB], (j / C::QB) & 1, p.err);
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_qk = idesc_bf16_f32(kTileM, C::BN, false, false);
    constexpr uint32_t idesc_pv = idesc_bf16_f32(kTileM, C::D, false, true);
    const uint32_t smem_base = smem_u32(smem);
    long long i = 0;
    int ux[2] = {0, 0};    // units started per tile (Q buffer index)
    int px[2] = {0, 0};    // P.V issued per tile (p_full phase)
    long long pend[2] = {-1, -1};  // key tile of the pending P.V per tile
    int pflags[2] = {0, 0};        // bit 0 first tile of the unit, bit 1 last
    uint32_t vusers = 0;           // per V stage (4 bits each): P.V still to read it
    auto issue_pv = [&](int x) {
      const long long j = pend[x];
      const int st = (int)(j % C::VST);
      mbar_wait(&p_full[x], px[x] & 1, p.err);
      mbar_wait(&v_full[st], (int)(j / C::VST) & 1, p.err);
      tc_fence_after();
      ++px[x];
      const uint32_t v_addr = smem_base + C::kOffV + st * C::kKVBytes;
      const bool first = pflags[x] & 1;
#pragma unroll
      for (int kk = 0; kk < C::BN / 16; ++kk) {
        const uint64_t bdesc = sw128_desc(v_addr + kk * 16 * 128, C::kKVBytes, 1024);
        mma_ts_w(tmem + C::col_o(x), tmem + C::col_s(x) + kk * 8, bdesc, idesc_pv, (kk > 0 || !first) ? 1u : 0u);
      }
      const uint32_t left = ((vusers >> (4 * st)) & 0xFu) - 1u;
      vusers = (vusers & ~(0xFu << (4 * st))) | (left << (4 * st));
      if (left == 0) mma_commit_w(&v_empty[st]);
      if (pflags[x] & 2) mma_commit_w(&o_full[x]);
      pend[x] = -1;
    };
    for (PairStream<C::BN> ps(p, blockIdx.x, n_pairs, gridDim.x, n_items); ps.valid(); ps.advance(p)) {
      const PairInfo& pi = ps.cur;
      if (pi.n == 0) continue;
      int jx[2] = {0, 0};
      for (int t = 0; t < pi.n; ++t, ++i) {
        int row, mask;
        stream_tile<C::BN>(pi, t, row, mask);
        const int st = (int)(i % C::ST);
        // A P.V pending for VST tiles holds the V stage the producer must refill before it can
        // issue this K tile: issue it first.
#pragma unroll
        for (int x = 0; x < 2; ++x)
          if (pend[x] >= 0 && pend[x] <= i - C::VST) issue_pv(x);
        // P.V still pending for a tile this key tile feeds must precede its QK (one S buffer);
        // issue them before waiting for the K copy so their epilogue never waits on it.
        if (!__all_sync(0xffffffffu, mbar_try_wait(&k_full[st], (int)(i / C::ST) & 1))) {
#pragma unroll
          for (int x = 0; x < 2; ++x)
            if ((mask >> x) & 1 && pend[x] >= 0) issue_pv(x);
        }
        mbar_wait(&k_full[st], (int)(i / C::ST) & 1, p.err);
        tc_fence_after();
        const uint32_t k_addr = smem_base + C::kOffK + st * C::kKVBytes;
        const int vst = (int)(i % C::VST);
        vusers = (vusers & ~(0xFu << (4 * vst))) | ((uint32_t)__popc(mask) << (4 * vst));
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (!((mask >> x) & 1)) continue;
          if (pend[x] >= 0) issue_pv(x);
          const int qb = ux[x] % C::QB;
          if (jx[x] == 0) {
            mbar_wait(&q_full[x * C::QB + qb], (ux[x] / C::QB) & 1, p.err);
            tc_fence_after();
          }
          const uint32_t q_addr = smem_base + C::kOffQ + (x * C::QB + qb) * C::kQBytes;
#pragma unroll
          for (int kk = 0; kk < C::D / 16; ++kk) {
            const uint64_t adesc = sw128_desc(q_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = sw128_desc(k_addr + kk * 32, 16, 1024);
            mma_ss_w(tmem + C::col_s(x), adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit_w(&s_full[x]);
          const bool last = jx[x] == pi.t[x].n_kv - 1;
          if (last) {
            mma_commit_w(&q_empty[x * C::QB + qb]);
            ++ux[x];
          }
          pend[x] = i;
          pflags[x] = (jx[x] == 0 ? 1 : 0) | (last ? 2 : 0);
          ++jx[x];
        }
        mma_commit_w(&k_empty[st]);
      }
    }
#pragma unroll
    for (int x = 0; x < 2; ++x)
      if (pend[x] >= 0) issue_pv(x);
  }  // warps 2-3: idle
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    constexpr int kCols = C::BN;  // S columns per thread per key tile (one row per thread)
    constexpr int kPass = C::kPass;  // S columns held in registers at once
    const int x = (warp - 4) >> 2;  // tile of this warp group
    const int sw = warp - 4;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row of this thread == TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + C::col_s(x);
    const uint32_t o_addr = tmem + lane_base + C::col_o(x);
    const float NEG_INF = -__int_as_float(0x7f800000);
    const float c2 = p.scale_log2;
    int sc = 0;  // key tiles processed (s_full / p_full phase)
    int uc = 0;  // units finished (o_full phase)
    // This group's tile of each pair: item 2 * (pair / heads) + x; the next schedule entry is
    // loaded one pair ahead.
    auto item_of = [&](long long pp) { return 2 * (pp / p.heads) + x; };
    long long pp = blockIdx.x;
    WorkItem nxt{};
    if (pp < n_pairs && item_of(pp) < n_items) nxt = p.items[item_of(pp)];
    for (; pp < n_pairs; pp += gridDim.x) {
      const long long item = item_of(pp);
      const WorkItem cur = nxt;
      const long long pn = pp + gridDim.x;
      if (pn < n_pairs && item_of(pn) < n_items) nxt = p.items[item_of(pn)];
      if (item >= n_items) continue;
      const UnitInfo ui = unit_info_from<C::BN>(p, cur, item * p.heads + pp % p.heads);
      if (ui.n_kv == 0) continue;
      const bool row_valid = r < ui.nq;
      const int tq = ui.q_row0 + r;
      int s = ui.f;
      if (ui.c > 1) {
        int cnt = 0;
        for (int base = 1; base < ui.c; base += 32) {
          const int idx = base + lane;
          const int v = idx < ui.c ? p.cu_q[ui.f + idx] : 0x7fffffff;
#pragma unroll 8
          for (int j = 0; j < 32; ++j) cnt += (__shfl_sync(0xffffffffu, v, j) <= tq) ? 1 : 0;
        }
        s = min(ui.f + cnt, ui.f + ui.c - 1);
      }
      int klo = 0, khi = 0;
      if (row_valid) {
        const int cq = p.cu_q[s], lq = p.cu_q[s + 1] - cq;
        const int ck = p.cu_k[s], lk = p.cu_k[s + 1] - ck;
        const int pos = tq - cq + (lk - lq);
        klo = ck + (p.window_left >= 0 ? max(0, pos - p.window_left) : 0);
        khi = ck + (p.window_right >= 0 ? min(lk, pos + p.window_right + 1) : lk);
      }
      float m_run = NEG_INF, l_run = 0.f;
      for (int t = 0; t < ui.n_kv; ++t, ++sc) {
        const int kt = ui.kv_lo + t * C::BN;
        const int c_lo = klo - kt, c_hi = khi - kt;
        const bool full = __all_sync(0xffffffffu, c_lo <= 0 && c_hi >= kCols);
        uint32_t active = 0;
#pragma unroll
        for (int cc = 0; cc < kCols / 32; ++cc)
          active |= (__any_sync(0xffffffffu, c_lo < 32 * (cc + 1) && c_hi > 32 * cc && c_lo < c_hi) ? 1u : 0u) << cc;
        mbar_wait(&s_full[x], sc & 1, p.err);
        tc_fence_after();
        // Pass 1: row max over kPass columns at a time (TMEM is re-read in pass 2 when the row
        // does not fit in registers).
        uint32_t raw[kPass];
        float mxs[4] = {NEG_INF, NEG_INF, NEG_INF, NEG_INF};
#pragma unroll
        for (int h = 0; h < kCols / kPass; ++h) {
#pragma unroll
          for (int cc = 0; cc < kPass / 32; ++cc)
            if (full || (active & (1u << (h * (kPass / 32) + cc))))
              tmem_ld32(s_addr + h * kPass + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&raw[cc * 32]));
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
                mxs[j & 3] = fmaxf(mxs[j & 3], ok ? __uint_as_float(raw[cc * 32 + j]) : NEG_INF);
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
        float2 accs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        // Pass 2: p = exp2(s * scale_log2 - m), bf16 pairs written over S, fp32 row sum.
#pragma unroll
        for (int h = 0; h < kCols / kPass; ++h) {
          if (kCols > kPass) {
#pragma unroll
            for (int cc = 0; cc < kPass / 32; ++cc)
              if (full || (active & (1u << (h * (kPass / 32) + cc))))
                tmem_ld32(s_addr + h * kPass + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(&raw[cc * 32]));
            tmem_wait_ld();
          }
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
#pragma unroll
          for (int cc = 0; cc < kPass / 32; ++cc) {
            uint32_t pk[16];
            if (full || (active & (1u << (h * (kPass / 32) + cc)))) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float2 xv = ffma2(
                    make_float2(__uint_as_float(raw[cc * 32 + 2 * j]), __uint_as_float(raw[cc * 32 + 2 * j + 1])), cc2,
                    nb2);
                const float2 e = make_float2(ex2(xv.x), ex2(xv.y));
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
        // O rescale (rare). S_X(t) was published after P.V_X(t-1) completed, so O is final.
        if (any_need) {
#pragma unroll
          for (int cc = 0; cc < C::D / 32; ++cc) {
            uint32_t o[32];
            tmem_ld32(o_addr + cc * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float2 v =
                  fmul2(make_float2(__uint_as_float(o[j]), __uint_as_float(o[j + 1])), make_float2(alpha, alpha));
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
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
      // Epilogue: O / l -> bf16 rows through a 2 KB per-warp stage (coalesced 64-byte row
      // segments), LSE in natural log.
      mbar_wait(&o_full[x], uc & 1, p.err);
      ++uc;
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint4* stage = reinterpret_cast<uint4*>(smem + C::kOffStage + sw * 2048);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t o[32];
        tmem_ld32(o_addr + hh * 32, o);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          pk[j] = pack_bf16x2(__uint_as_float(o[2 * j]) * inv, __uint_as_float(o[2 * j + 1]) * inv);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          stage[lane * 4 + (c ^ ((lane >> 1) & 3))] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int row = k * 8 + (lane >> 2), c = lane & 3;
          uint4 val = stage[row * 4 + (c ^ ((row >> 1) & 3))];
          const int tr = quarter * 32 + row;
          const int tok = ui.q_row0 + tr;
          if (tr < ui.nq && tok < p.total_q) {
            store_out(reinterpret_cast<uint4*>(p.out + (long long)tok * p.o_tok + (long long)ui.head * p.o_head +
                                               hh * 32 + c * 8),
                      val);
          }
        }
        __syncwarp();
      }
      if (row_valid && tq < p.total_q && p.lse != nullptr) {
        const float lse = l_run > 0.f ? (m_run + __log2f(l_run)) * 0.69314718055994531f : NEG_INF;
        p.lse[(long long)ui.head * p.total_q + tq] = lse;
      }
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}
