// One CTA per search lane, one action per thread (W = ceil(A / 32) warps);
// the heavy per-(action, sample) and per-(action, grid point) cells of the
// estimators are spread over all threads through a compacted action list.
//
// The descent and the bottom-up repair walk a lane's tree one node at a
// time, so their latency per node bounds the whole launch: a few deep lanes
// finish long after the rest.  Spreading a node's actions over W warps cuts
// that latency by W against the warp-per-lane mapping.  Reductions over
// actions keep the canonical order (partial sums v[t] + v[t+32] + v[t+64] +
// v[t+96], then the xor butterfly), computed by warp 0 from shared memory.
//
// The quadrature grid's per-(action, point) values live in shared-memory
// matrices [Q][32W] so each grid point's sum over actions is one warp's
// column reduction, and the estimator's guards are evaluated after the
// density normalisation: when they already force the Monte Carlo fallback,
// the remaining prefix-CDF passes are skipped (their policy is discarded).
//
// Included inside search.cu's anonymous namespace.

template <int W>
struct Cta {
  static constexpr int kT = 32 * W;
  float *red;        // [2][kT] reduction inputs
  float *bc;         // [16] broadcast results
  float *pv;         // [W] per-warp argmax values
  int *pi;           // [W] per-warp argmax indices
  float *lx, *l1mx, *lj, *flp, *joint, *score;  // [Q]
  float *zc;         // [Q] zero counts (exact small integers)
  float *D, *F;       // [Qs][kT]; the Monte Carlo population reuses them for [kKeyChunk][kT] utilities
  uint8_t *Z;         // [Qs][kT] zero-CDF flags
  DrawKeys *keys;     // [kKeyChunk] derived keys of a chunk of samples
  int *best;          // [kKeyChunk] argmax of each sample of a chunk
  float4 *shape;      // [2][kT] Gamma constants of the compacted sampled actions (shares Z's storage)
  int *live;          // [kT] compacted list of the actions that carry work
  float *ascale, *asafe;  // [kT] per-action density shift and normaliser
  float *zint, *jinc;     // [Q] integrand of a non-unresolved action; joint increments
  int Q;
};

constexpr int kKeyChunk = 16;

// matrix rows: enough for Q grid points and, over D and F together, for a
// chunk of sample utilities (kKeyChunk rows), their second variates
// (kKeyChunk rows) and the redraw list (kKeyChunk rows of 16-bit pairs)
__host__ __device__ constexpr int cta_rows(int Q) { return Q > 3 * kKeyChunk / 2 ? Q : 3 * kKeyChunk / 2; }

// The Monte Carlo draw's Gamma constants (8 kT floats) and the quadrature's
// zero-CDF flags (rows x kT bytes) are never live in the same pass of a node
// update, so they share one region.
template <int W>
__host__ __device__ constexpr size_t cta_shared_region_floats(int Q) {
  return (size_t)8 * Cta<W>::kT > ((size_t)cta_rows(Q) * Cta<W>::kT + 3) / 4
             ? (size_t)8 * Cta<W>::kT
             : ((size_t)cta_rows(Q) * Cta<W>::kT + 3) / 4;
}

template <int W>
__host__ __device__ constexpr size_t cta_smem_floats(int Q) {
  return cta_shared_region_floats<W>(Q) + (size_t)2 * Cta<W>::kT + 16 + 2 * W + kKeyChunk +
         (size_t)kKeyChunk * (sizeof(DrawKeys) / sizeof(float)) + 3 * (size_t)Cta<W>::kT + 9 * (size_t)Q +
         2 * (size_t)cta_rows(Q) * Cta<W>::kT;
}

template <int W>
__device__ __forceinline__ Cta<W> cta_scratch(int Q) {
  extern __shared__ __align__(16) float smem[];
  Cta<W> c;
  float *p = smem;
  c.shape = reinterpret_cast<float4 *>(p);  // first: 16-byte aligned
  c.Z = reinterpret_cast<uint8_t *>(p);
  p += cta_shared_region_floats<W>(Q);
  c.red = p;
  p += 2 * Cta<W>::kT;
  c.bc = p;
  p += 16;
  c.pv = p;
  p += W;
  c.pi = reinterpret_cast<int *>(p);
  p += W;
  c.best = reinterpret_cast<int *>(p);
  p += kKeyChunk;
  c.keys = reinterpret_cast<DrawKeys *>(p);
  p += kKeyChunk * (sizeof(DrawKeys) / sizeof(float));
  c.lx = p;
  c.l1mx = p + Q;
  c.lj = p + 2 * Q;
  c.flp = p + 3 * Q;
  c.joint = p + 4 * Q;
  c.score = p + 5 * Q;
  c.zc = p + 6 * Q;
  c.zint = p + 7 * Q;
  c.jinc = p + 8 * Q;
  p += 9 * Q;
  c.live = reinterpret_cast<int *>(p);
  c.ascale = p + Cta<W>::kT;
  c.asafe = p + 2 * Cta<W>::kT;
  p += 3 * Cta<W>::kT;
  const size_t m = (size_t)cta_rows(Q) * Cta<W>::kT;
  c.D = p;
  c.F = p + m;
  c.Q = Q;
  return c;
}

// canonical sum of column `col` (length A) of a [*, kT] matrix, by one warp
template <int W>
__device__ __forceinline__ float column_sum(const float *col, int A, int lane) {
  float p = 0.0f;
  bool first = true;
#pragma unroll
  for (int j = 0; j < W; ++j) {
    const int a = lane + kWarp * j;
    if (a < A) {
      p = first ? col[a] : p + col[a];
      first = false;
    }
  }
  return butterfly_sum(p);
}

// canonical sum over actions of the clipped log-CDF of column `col`:
// -inf where the CDF is zero (z set), else min(log CDF, 0)
template <int W>
__device__ __forceinline__ float column_sum_clipped(const float *f, const uint8_t *z, int A, int lane) {
  float p = 0.0f;
  bool first = true;
#pragma unroll
  for (int j = 0; j < W; ++j) {
    const int a = lane + kWarp * j;
    if (a < A) {
      const float fv = f[a];
      const float x = z[a] ? -SM_INF : (fv < 0.0f ? fv : 0.0f);
      p = first ? x : p + x;
      first = false;
    }
  }
  return butterfly_sum(p);
}

// The cells t, t + T, t + 2T, ... of a grid with n cells per row, as
// (row, column) pairs: two divisions per walk instead of one per cell.
// With n = 0 the grid is empty and the walk starts past every row.
struct CellWalk {
  int row, col, drow, dcol;
  __device__ __forceinline__ CellWalk(int t, int T, int n) {
    const int m = n > 0 ? n : 1;
    row = n > 0 ? t / m : INT_MAX;
    col = t - (n > 0 ? row : 0) * m;
    drow = T / m;
    dcol = T - drow * m;
  }
  __device__ __forceinline__ void next(int n) {
    col += dcol;
    row += drow;
    if (col >= n) {
      col -= n;
      row += 1;
    }
  }
};

// Up to 4 simultaneous canonical sums over actions; every thread gets them.
template <int W, int K>
__device__ __forceinline__ void cta_sums(const Cta<W> &c, const float (&v)[K], float (&out)[K], int A) {
  const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
#pragma unroll
  for (int k = 0; k < K; ++k) c.red[k * Cta<W>::kT + t] = v[k];
  __syncthreads();
  for (int kk = warp; kk < K; kk += W) {
    const float s = column_sum<W>(c.red + kk * Cta<W>::kT, A, lane);
    if (lane == 0) c.bc[kk] = s;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < K; ++k) out[k] = c.bc[k];
  __syncthreads();
}

template <int W>
__device__ __forceinline__ float cta_sum(const Cta<W> &c, float v, int A) {
  float in[1] = {v}, out[1];
  cta_sums<W, 1>(c, in, out, A);
  return out[0];
}

// argmax over a per-thread value (thread index = action index), with the
// jnp.argmax order of `beats`
template <int W>
__device__ __forceinline__ int cta_argmax_by_action(const Cta<W> &c, float v, int A) {
  const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
  const float vv = t < A ? v : -SM_INF;
  const int ii = t < A ? t : INT_MAX;
  c.red[Cta<W>::kT + t] = vv;
  const int wi = warp_argmax(vv, ii);
  if (lane == 0) c.pi[warp] = wi;
  __syncthreads();
  float bv = -SM_INF;
  int bi = INT_MAX;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const int i = c.pi[w];
    const float val = i == INT_MAX ? -SM_INF : c.red[Cta<W>::kT + i];
    if (beats(val, i, bv, bi)) {
      bv = val;
      bi = i;
    }
  }
  __syncthreads();
  return bi;
}

template <int W>
__device__ __forceinline__ int cta_reduce_add(const Cta<W> &c, int v) {
  const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
  const int s = __reduce_add_sync(kFull, v);
  if (lane == 0) c.pi[warp] = s;
  __syncthreads();
  int total = 0;
#pragma unroll
  for (int w = 0; w < W; ++w) total += c.pi[w];
  __syncthreads();
  return total;
}

template <int W>
__device__ __forceinline__ int cta_reduce_min(const Cta<W> &c, int v) {
  const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
  const int s = __reduce_min_sync(kFull, v);
  if (lane == 0) c.pi[warp] = s;
  __syncthreads();
  int m = c.pi[0];
#pragma unroll
  for (int w = 1; w < W; ++w) m = c.pi[w] < m ? c.pi[w] : m;
  __syncthreads();
  return m;
}

template <int W>
__device__ __forceinline__ int cta_reduce_max(const Cta<W> &c, int v) {
  const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
  const int s = __reduce_max_sync(kFull, v);
  if (lane == 0) c.pi[warp] = s;
  __syncthreads();
  int m = c.pi[0];
#pragma unroll
  for (int w = 1; w < W; ++w) m = c.pi[w] > m ? c.pi[w] : m;
  __syncthreads();
  return m;
}

// exact float min/max (order independent; NaN never wins, as in the oracle)
template <int W>
__device__ __forceinline__ float cta_min_float(const Cta<W> &c, float v) {
  const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
  const float s = warp_min_float(v);
  if (lane == 0) c.pv[warp] = s;
  __syncthreads();
  float m = c.pv[0];
#pragma unroll
  for (int w = 1; w < W; ++w) m = c.pv[w] < m ? c.pv[w] : m;
  __syncthreads();
  return m;
}

template <int W>
__device__ __forceinline__ float cta_max_float(const Cta<W> &c, float v) {
  const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
  const float s = warp_max_float(v);
  if (lane == 0) c.pv[warp] = s;
  __syncthreads();
  float m = c.pv[0];
#pragma unroll
  for (int w = 1; w < W; ++w) m = c.pv[w] > m ? c.pv[w] : m;
  __syncthreads();
  return m;
}

__device__ __forceinline__ float draw_utility(const DrawKeys &k, const GammaShape &g0, const GammaShape &g1,
                                              uint64_t base, uint64_t stride);

// thompson_sample (action_selection.py:135-143) with one action per thread
template <int W>
__device__ int cta_thompson(const Cta<W> &c, const DrawKeys &k, const GammaShape &g0, const GammaShape &g1,
                            bool masked, int8_t cat, bool use_cat, int A, uint64_t lane_base, uint64_t stride) {
  const int a = threadIdx.x;
  float u = -SM_INF;
  if (a < A && !masked) {
    if (use_cat && cat != kNoOutcome) {
      u = cat == 1 ? 1.0f : (cat == 0 ? -1.0f : 0.0f);
    } else {
      u = draw_utility(k, g0, g1, lane_base + (uint64_t)a * 2u, stride);
    }
  }
  return cta_argmax_by_action<W>(c, u, A);
}

// the three draw keys of one Thompson sample, derived by one thread
template <int W>
__device__ __forceinline__ DrawKeys cta_draw_keys(const Cta<W> &c, sk_key key) {
  if (threadIdx.x == 0) c.keys[0] = draw_keys(key);
  __syncthreads();
  const DrawKeys k = c.keys[0];
  __syncthreads();
  return k;
}

// exact utility of a categorical edge (outcomes.py:38-43)
__device__ __forceinline__ float categorical_utility(int8_t cat) {
  return cat == 1 ? 1.0f : (cat == 0 ? -1.0f : 0.0f);
}

// utility of one Thompson draw of this thread's action
__device__ __forceinline__ float draw_utility(const DrawKeys &k, const GammaShape &g0, const GammaShape &g1,
                                              uint64_t base, uint64_t stride) {
  const float lg0 = log_gamma_draw(k, base, stride, g0);
  const float lg1 = log_gamma_draw(k, base + 1, stride, g1);
  return binary_utility(lg0, lg1);
}

// Two CTA-wide ORs and a float maximum (as cta_max_float) behind one barrier.
template <int W>
__device__ __forceinline__ float cta_guards(const Cta<W> &c, bool f1, bool f2, float v, bool &any1, bool &any2) {
  const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
  const unsigned b1 = __ballot_sync(kFull, f1), b2 = __ballot_sync(kFull, f2);
  const float m = warp_max_float(v);
  if (lane == 0) {
    c.pi[warp] = (b1 != 0u ? 1 : 0) | (b2 != 0u ? 2 : 0);
    c.pv[warp] = m;
  }
  __syncthreads();
  int f = 0;
  float r = c.pv[0];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    f |= c.pi[w];
    if (w > 0) r = c.pv[w] > r ? c.pv[w] : r;
  }
  __syncthreads();
  any1 = (f & 1) != 0;
  any2 = (f & 2) != 0;
  return r;
}

// Everything a node update reduces over its actions that is known once the
// actions are gathered, in one pass: per-warp ballots and warp reductions,
// one barrier, then every thread combines the W warps' partials.  The
// results are integers, flags and an exact minimum, identical to separate
// CTA reductions.  It also lists the unresolved legal actions in c.live in
// increasing order: the estimators spread their per-(action, grid point)
// and per-(action, sample) cells over all threads by position in that list,
// so illegal and resolved actions leave no thread idle.
struct NodeSummary {
  int n_unres;       // unresolved legal actions (the length of c.live)
  int slot;          // this thread's position in c.live, if it is listed
  int delta;         // sum of the payload changes of the unresolved legal actions
  bool has_legal, has_win;
  int shortest_win;  // min payload over certified wins (INT_MAX if none)
  int longest_loss;  // max payload over certified losses (INT_MIN if none)
  int first_win;     // lowest certified winning action (INT_MAX if none)
  float amin;        // min over unresolved of min(max(alpha, tiny)) per outcome
  int visited;       // actions with a visited child (statistics only)
};

template <int W>
__device__ __forceinline__ NodeSummary cta_node_summary(const Cta<W> &c, bool legal, bool unres, bool win, bool loss,
                                                        int delta, int payload, float amin, bool visited) {
  const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
  const unsigned mu = __ballot_sync(kFull, unres), ml = __ballot_sync(kFull, legal);
  const unsigned mw = __ballot_sync(kFull, win), mv = __ballot_sync(kFull, visited);
  const int d = __reduce_add_sync(kFull, delta);
  const int sw = __reduce_min_sync(kFull, win ? payload : INT_MAX);
  const int ll = __reduce_max_sync(kFull, loss ? payload : INT_MIN);
  const int fw = __reduce_min_sync(kFull, win ? t : INT_MAX);
  const float am = warp_min_float(amin);
  int *wi = reinterpret_cast<int *>(c.red);  // [W][8], then [W] floats
  float *wf = c.red + 8 * W;
  if (lane == 0) {
    wi[warp * 8 + 0] = __popc(mu);
    wi[warp * 8 + 1] = ml != 0u;
    wi[warp * 8 + 2] = mw != 0u;
    wi[warp * 8 + 3] = d;
    wi[warp * 8 + 4] = sw;
    wi[warp * 8 + 5] = ll;
    wi[warp * 8 + 6] = fw;
    wi[warp * 8 + 7] = __popc(mv);
    wf[warp] = am;
  }
  __syncthreads();
  NodeSummary r;
  r.n_unres = 0;
  r.delta = 0;
  r.has_legal = false;
  r.has_win = false;
  r.shortest_win = INT_MAX;
  r.longest_loss = INT_MIN;
  r.first_win = INT_MAX;
  r.amin = wf[0];
  r.visited = 0;
  int off = 0;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const int *q = wi + w * 8;
    off += w < warp ? q[0] : 0;
    r.n_unres += q[0];
    r.has_legal |= q[1] != 0;
    r.has_win |= q[2] != 0;
    r.delta += q[3];
    r.shortest_win = q[4] < r.shortest_win ? q[4] : r.shortest_win;
    r.longest_loss = q[5] > r.longest_loss ? q[5] : r.longest_loss;
    r.first_win = q[6] < r.first_win ? q[6] : r.first_win;
    r.visited += q[7];
    if (w > 0) r.amin = wf[w] < r.amin ? wf[w] : r.amin;
  }
  r.slot = off + __popc(mu & ((1u << lane) - 1u));
  if (unres) c.live[r.slot] = t;
  __syncthreads();
  return r;
}

// Utilities U[s][action] of samples s < n of a chunk for the ns compacted
// sampled actions (their Gamma constants in c.shape), in four passes over
// cells so that the rare branches of the Marsaglia-Tsang draw do not hold
// whole warps: (1) the first proposal of both variates of every cell;
// (2) the full draw for the variates whose first proposal was rejected,
// from a list; (3) the alpha < 1 augmentation for the (action, outcome)
// pairs listed in `aug`; (4) the utility.  Each variate goes through exactly
// the operations of log_gamma_draw, so the values equal a per-cell draw.
// GU unrolls the two variates of pass (1): 2 measured faster in the Monte
// Carlo kernel, 1 (less code next to the quadrature) in the prefix-CDF one.
template <int W, int GU>
__device__ void cta_draw_chunk(const Cta<W> &c, int n, int ns, const int *aug, int na, uint64_t lane_base,
                               uint64_t stride) {
  constexpr int T = Cta<W>::kT;
  const int a = threadIdx.x;
  float *const L[2] = {c.D, c.D + kKeyChunk * T};  // [kKeyChunk][T] each; L[0] becomes U
  uint16_t *redo = reinterpret_cast<uint16_t *>(c.D + 2 * kKeyChunk * T);  // 2 * kKeyChunk * T entries
  for (CellWalk w(a, T, ns); w.row < n; w.next(ns)) {
    const int s = w.row, slot = w.col;
    const int aa = c.live[slot];
    const uint64_t base = lane_base + (uint64_t)aa * 2u;
#pragma unroll GU
    for (int g = 0; g < 2; ++g) {
      const float4 p = c.shape[2 * slot + g];
      float v;
      if (gamma_first(c.keys[s], base + g, p.y, p.z, p.w, v))
        L[g][s * T + aa] = v;
      else
        redo[atomicAdd(&c.pi[0], 1)] = (uint16_t)((s << 8) | (slot << 1) | g);
    }
  }
  __syncthreads();
  const int nr = c.pi[0];
  for (int e = a; e < nr; e += T) {
    const int code = redo[e], s = code >> 8, slot = (code >> 1) & 127, g = code & 1;
    const int aa = c.live[slot];
    const float4 p = c.shape[2 * slot + g];
    const GammaShape gs = {p.x, p.y, p.z, p.w};
    L[g][s * T + aa] = log_gamma_core(c.keys[s], lane_base + (uint64_t)aa * 2u + g, stride, gs);
  }
  __syncthreads();
  for (CellWalk w(a, T, na); w.row < n; w.next(na)) {
    const int s = w.row, code = aug[w.col], slot = code >> 1, g = code & 1;
    const int aa = c.live[slot];
    float &lg = L[g][s * T + aa];
    lg = gamma_augment(c.keys[s], lane_base + (uint64_t)aa * 2u + g, c.shape[2 * slot + g].x, lg);
  }
  __syncthreads();
  for (CellWalk w(a, T, ns); w.row < n; w.next(ns)) {
    const int s = w.row, aa = c.live[w.col];
    L[0][s * T + aa] = binary_utility(L[0][s * T + aa], L[1][s * T + aa]);
  }
}

// posterior_best_policy (action_selection.py:146-194).  The utilities of a
// chunk of samples are drawn cell by cell over (sample, sampled action),
// every thread taking cells in turn; warps then take one sample's argmax
// each, and each thread counts its own action's hits.
// Categorical edges take their exact utility, so the sampled actions are
// exactly the node's unresolved legal ones: the summary's c.live list.
template <int W, int GU>
__device__ float cta_mc_policy(const Cta<W> &c, const NodeSummary &sum, sk_key key, float a0, float a1, bool invalid,
                               int8_t cat, int S, int A, int b, int B) {
  constexpr int T = Cta<W>::kT;
  const int a = threadIdx.x, lane = a % kWarp, warp = a / kWarp;
  const bool present = a < A;
  const bool exact = present && !invalid && cat != kNoOutcome;
  const bool sampled = present && !invalid && !exact;
  const uint64_t lane_base = (uint64_t)b * A * 2u, stride = (uint64_t)B * A * 2u;
  const int slot = sum.slot, ns = sum.n_unres;
  // Gamma constants by slot, and the list of (slot, outcome) variates whose
  // concentration is below 1 (they take the augmentation)
  int *aug = reinterpret_cast<int *>(c.red);  // up to 2 * T entries
  if (a == 0) c.pi[0] = 0;
  __syncthreads();
  if (sampled) {
    const GammaShape g0 = gamma_shape(a0), g1 = gamma_shape(a1);
    c.shape[2 * slot] = make_float4(g0.alpha, g0.d, g0.c, g0.logd);
    c.shape[2 * slot + 1] = make_float4(g1.alpha, g1.d, g1.c, g1.logd);
    if (g0.alpha < 1.0f) aug[atomicAdd(&c.pi[0], 1)] = 2 * slot;
    if (g1.alpha < 1.0f) aug[atomicAdd(&c.pi[0], 1)] = 2 * slot + 1;
  }
  __syncthreads();
  const int na = c.pi[0];
  const float fixed = exact ? categorical_utility(cat) : -SM_INF;
  // one sample draws with `key` itself; more samples split(split(key)[0], S)
  const sk_key sample_key = sk_split(key, 0);
  int hits = 0;
  float *U = c.D;  // [kKeyChunk][T]
  for (int s0 = 0; s0 < S; s0 += kKeyChunk) {
    const int n = S - s0 < kKeyChunk ? S - s0 : kKeyChunk;
    __syncthreads();  // the previous chunk's (or the list's) counter reads are done
    if (a == 0) c.pi[0] = 0;
    if (a < n) c.keys[a] = draw_keys(S == 1 ? key : sk_split(sample_key, (uint64_t)(s0 + a)));
    if (!sampled)
      for (int s = 0; s < n; ++s) U[s * T + a] = fixed;
    __syncthreads();
    cta_draw_chunk<W, GU>(c, n, ns, aug, na, lane_base, stride);
    __syncthreads();
    for (int s = warp; s < n; s += W) {
      float bv = -SM_INF;
      int bi = INT_MAX;
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const int aa = lane + kWarp * j;
        if (aa < A && beats(U[s * T + aa], aa, bv, bi)) {
          bv = U[s * T + aa];
          bi = aa;
        }
      }
      const int w = warp_argmax(bv, bi);
      if (lane == 0) c.best[s] = w;
    }
    __syncthreads();
    for (int s = 0; s < n; ++s) hits += c.best[s] == a;
    __syncthreads();
  }
  if (S == 1) return (present && !invalid && hits) ? 1.0f : 0.0f;
  const int legal = __syncthreads_count(present && !invalid);
  float policy = (present && !invalid) ? (float)hits / (float)S : 0.0f;
  const float total = cta_sum<W>(c, policy, A);
  const float denom = total > 1.0f ? total : 1.0f;
  const float lc = (float)(legal > 1 ? legal : 1);
  return total > 0.0f ? policy / denom : (invalid ? 0.0f : 1.0f) / lc;
}

struct PrefixResult1 {
  float policy;  // this thread's action
  bool unsafe;   // clipped, non-finite or density error above tolerance
};

// binary_posterior_best_policy_prefix_quadrature (prefix_cdf.py:217-445) and
// the guard of update_posterior_prefix_cdf (posterior_updates.py:282-290).
// Running sums over grid points (trapezoid integrals, the policy's sum over
// intervals) are taken by each action's own thread in grid order; the
// transcendental work per (unresolved action, grid point) cell is spread
// over all threads by the compacted list of unresolved actions.  Each cell
// evaluates exactly the expression of the per-action loop, so the result
// does not depend on the mapping.  Returns early with unsafe = true as soon
// as the clipping or density guard fires.
template <int W>
__device__ PrefixResult1 cta_prefix_guarded(const Cta<W> &c, const NodeSummary &sum, float a0, float a1, bool invalid,
                                            int8_t outc, int A, const PrefixParams &P, float tol) {
  const int a = threadIdx.x, lane = a % kWarp, warp = a / kWarp;
  const int h = P.h, Q = 2 * h + 1;
  const int T = Cta<W>::kT;
  const bool present = a < A;
  const bool legal = present && !invalid;
  const bool unres = legal && outc == kNoOutcome;
  const int n_unres = sum.n_unres;
  const bool has_unres = n_unres > 0;
  const bool has_legal = sum.has_legal;
  const bool has_cw = sum.has_win;
  const float amin = sum.amin;
  float requested = sm_asinhf_pos(P.tail / amin);
  if (!has_unres) requested = P.min_hr;
  float hr = requested;
  if (hr < P.min_hr) hr = P.min_hr;
  if (hr > P.max_hr) hr = P.max_hr;
  const bool clipped = has_unres && requested > P.max_hr;
  PrefixResult1 r;
  r.policy = 0.0f;
  r.unsafe = clipped;
  if (clipped) return r;
  const float fh = (float)h;
  for (int k = a; k < Q; k += T) {
    const float unit = (float)(k - h) / fh;
    const float coord = hr * unit;
    const float logit = sm_sinhf(coord);
    c.lx[k] = -sm_softplusf(-logit);
    c.l1mx[k] = -sm_softplusf(logit);
    c.lj[k] = log_cosh(coord);
  }
  __syncthreads();
  const float hstep = 0.5f * (hr / fh);
  // log-density of this action on the grid; a resolved or illegal action
  // has density 0 everywhere (so zero CDF and no log-CDF contribution)
  bool nan = false;
  if (unres) {
    const float w = a1 > SM_TINY ? a1 : SM_TINY;
    const float l = a0 > SM_TINY ? a0 : SM_TINY;
    const float bl = sm_betalnf(w, l);
    float scale = -SM_INF;
    for (int k = 0; k < Q; ++k) {
      const float ld = ((w * c.lx[k] + l * c.l1mx[k]) - bl) + c.lj[k];
      c.D[k * T + a] = ld;
      nan |= ld != ld;
      if (ld > scale) scale = ld;
    }
    c.ascale[a] = nan ? SM_NAN : scale;
  } else {
    for (int k = 0; k < Q; ++k) {
      c.D[k * T + a] = 0.0f;
      c.F[k * T + a] = 0.0f;
      c.Z[k * T + a] = 0;
    }
  }
  __syncthreads();
  for (CellWalk w(a, T, n_unres); w.row < Q; w.next(n_unres)) {
    const int k = w.row, aa = c.live[w.col];
    c.D[k * T + aa] = sm_expf(c.D[k * T + aa] - c.ascale[aa]);
  }
  __syncthreads();
  // trapezoid running integral (kept in F until the CDF pass)
  float run = 0.0f;
  if (unres) {
    float prev = 0.0f;
    for (int k = 0; k < Q; ++k) {
      const float d = c.D[k * T + a];
      if (k > 0) run = run + hstep * (prev + d);
      prev = d;
      c.F[k * T + a] = run;
    }
  }
  const float dli = unres ? c.ascale[a] + sm_logf(run) : 0.0f;
  const float safe = run > 0.0f ? run : 1.0f;
  c.asafe[a] = safe;
  // guards available now: non-finite log-integral or |log-integral| > tol
  const float adli = fabsf(dli);
  bool dnan, dinf;
  const float derr = cta_guards<W>(c, present && adli != adli, unres && !sm_isfinite(dli), present ? adli : 0.0f,
                                   dnan, dinf);
  if (dinf || (!dnan && derr > tol)) {
    r.unsafe = true;
    return r;
  }
  // per grid point: CDF, its log and the zero-CDF flag (the clipped log-CDF
  // of the joint is formed from the two in the column sums)
  for (CellWalk w(a, T, n_unres); w.row < Q; w.next(n_unres)) {
    const int k = w.row, aa = c.live[w.col];
    const float cd = c.F[k * T + aa] / c.asafe[aa];
    const bool pos = cd > 0.0f;
    c.F[k * T + aa] = pos ? sm_logf(cd) : 0.0f;
    c.Z[k * T + aa] = pos ? 0 : 1;
  }
  __syncthreads();
  // leave-one-out products and the joint maximum CDF
  for (int k = warp; k < Q; k += W) {
    const float flp = column_sum<W>(c.F + k * T, A, lane);
    const float lsum = column_sum_clipped<W>(c.F + k * T, c.Z + k * T, A, lane);
    int zl = 0;
#pragma unroll
    for (int j = 0; j < W; ++j) zl += lane + kWarp * j < A ? c.Z[k * T + lane + kWarp * j] : 0;
    const float z = (float)__reduce_add_sync(kFull, zl);
    if (lane == 0) {
      c.flp[k] = flp;
      c.joint[k] = sm_expf(lsum);
      c.zc[k] = z;
    }
  }
  __syncthreads();
  if (a == 0) {
    c.joint[0] = has_unres ? 0.0f : 1.0f;
    c.joint[Q - 1] = 1.0f;
    for (int k = 1; k < Q; ++k) {
      const float p = c.joint[k - 1], cur = c.joint[k];
      if (p != p || (cur == cur && p > cur)) c.joint[k] = p;
    }
    c.joint[Q - 1] = 1.0f;
  }
  // winner integrand per (action, grid point); an action with zero density
  // (d = 0, CDF 0, normaliser 1) has the same integrand at every point
  for (int k = a; k < Q; k += T) {
    const float olp = (int)c.zc[k] > 0 ? -SM_INF : c.flp[k] - 0.0f;
    c.zint[k] = (0.0f / 1.0f) * sm_expf(olp);
  }
  for (CellWalk w(a, T, n_unres); w.row < Q; w.next(n_unres)) {
    const int k = w.row, aa = c.live[w.col];
    const float d = c.D[k * T + aa];
    const int zf = c.Z[k * T + aa];
    const float f = c.F[k * T + aa];
    const float olp = ((int)c.zc[k] - zf) > 0 ? -SM_INF : c.flp[k] - f;
    c.D[k * T + aa] = (d / c.asafe[aa]) * sm_expf(olp);
  }
  __syncthreads();
  // interval contributions (trapezoid of the integrand), clamped at 0; the
  // log-CDF rows are no longer read, so F holds them
  for (int k = 1; k < Q; ++k) {
    const float i0 = unres ? c.D[(k - 1) * T + a] : c.zint[k - 1];
    const float i1 = unres ? c.D[k * T + a] : c.zint[k];
    const float cc = hstep * (i0 + i1);
    c.F[(k - 1) * T + a] = cc > 0.0f ? cc : (cc != cc ? cc : 0.0f);
  }
  for (int j = a; j < Q - 1; j += T) {
    const float jinc = c.joint[j + 1] - c.joint[j];
    c.jinc[j] = jinc > 0.0f ? jinc : (jinc != jinc ? jinc : 0.0f);
  }
  __syncthreads();
  for (int j = warp; j < Q - 1; j += W) {
    const float sc = column_sum<W>(c.F + j * T, A, lane);
    if (lane == 0) c.score[j] = sc;
  }
  __syncthreads();
  // allocate each interval's joint increment in proportion to the
  // contributions (uniformly over unresolved actions if they sum to 0)
  const float uden = (float)(n_unres > 1 ? n_unres : 1);
  for (CellWalk w(a, T, n_unres); w.row < Q - 1; w.next(n_unres)) {
    const int j = w.row, aa = c.live[w.col];
    const float sc = c.score[j];
    const float wgt = sc > 0.0f ? c.F[j * T + aa] / sc : 1.0f / uden;
    c.D[j * T + aa] = wgt * c.jinc[j];
  }
  __syncthreads();
  float prob = 0.0f;
  if (unres)
    for (int j = 0; j < Q - 1; ++j) prob = prob + c.D[j * T + a];
  // _finalize_policy, prefix_cdf.py:121-183
  const int first_cw = sum.first_win;
  const float cs = legal ? (float)outc : -SM_INF;
  const int cbest = has_cw ? first_cw : cta_argmax_by_action<W>(c, cs, A);
  float raw = (has_cw || !has_unres) ? (a == cbest ? 1.0f : 0.0f) : (unres ? prob : 0.0f);
  raw = legal ? raw : 0.0f;
  const float mass = cta_sum<W>(c, raw, A);
  const float nerr = fabsf(mass - (has_legal ? 1.0f : 0.0f));
  const float smass = mass > 0.0f ? mass : 1.0f;
  float p = raw / smass;
  p = has_legal ? p : 0.0f;
  const bool fin_local = !present || (sm_isfinite(p) && sm_isfinite(raw));
  const bool finite = __syncthreads_and(fin_local) && sm_isfinite(mass) && sm_isfinite(nerr) && sm_isfinite(hr);
  r.policy = p;
  r.unsafe = !finite;
  return r;
}

// simulate / _simulate_one (search.py:21-78), one CTA per lane
template <int W>
__global__ void __launch_bounds__(32 * W) simulate_cta_kernel(Tree T, const uint32_t *key, int max_depth,
                                                              int32_t *out_parent, int32_t *out_action,
                                                              uint8_t *out_active, uint8_t *parent_emb,
                                                              unsigned long long *stats) {
  const int b = blockIdx.x, a = threadIdx.x;
  const Cta<W> c = cta_scratch<W>(1);
  const int A = T.A;
  const bool present = a < A;
  const sk_key sim_key = {key[0], key[1]};
  sk_key k = sk_split(sim_key, (uint64_t)b);
  // A node's row -- its player, its categorical outcome and this thread's
  // edge -- is loaded in one round, as soon as the node is known: the
  // searchable test of a child and the next level's draw then share it,
  // so a level waits for one round of dependent loads instead of two.
  int row_tp = 0, row_child = -1, row_payload = 0;
  int8_t row_outcome = kNoOutcome;
  bool row_masked = true;
  float2 row_alpha = make_float2(1.0f, 1.0f);
  auto load_row = [&](int n) {
    const size_t ni = T.node(b, n);
    row_tp = T.to_play[ni];
    row_outcome = T.node_outcome[ni];
    if (present) {
      const size_t e = T.edge(b, n, a);
      row_masked = T.invalid[e] || T.edge_outcome[e] != kNoOutcome;
      row_child = T.children[e];
      row_payload = T.edge_payload[e];
      row_alpha = T.edge_alpha[e];
    }
  };
  // any searchable edge: legal and not categorical
  auto searchable = [&]() { return __syncthreads_or(present && !row_masked) != 0; };
  load_row(0);
  const bool root_active = row_outcome == kNoOutcome && searchable();
  int node = 0, next = 0, action = 0, depth = 0;
  bool cont = root_active;
  const uint64_t stride = (uint64_t)A * 2u;
  unsigned long long visited_nodes = 0;
  int prior_gathers = 0;
  while (cont) {
    visited_nodes += 1;
    const sk_key next_key = sk_split(k, 0), sel_key = sk_split(k, 1);
    node = next;
    const int player = row_tp;
    bool masked = true;
    GammaShape g0 = gamma_shape(1.0f), g1 = g0;
    if (present) {
      masked = row_masked;
      if (!masked) {
        const int child = row_child;
        float2 alpha;
        if (child != -1 && row_payload <= 0 && T.ok(child)) {
          const size_t ci = T.node(b, child);
          alpha = align2(T.value_prior[ci], T.to_play[ci], player);
          prior_gathers += 1;
        } else {
          alpha = row_alpha;
        }
        g0 = gamma_shape(alpha.x);
        g1 = gamma_shape(alpha.y);
      }
    }
    action = cta_thompson<W>(c, cta_draw_keys<W>(c, sel_key), g0, g1, masked, kNoOutcome, false, A, 0, stride);
    int child = T.children[T.edge(b, node, action)];
    if (child != -1 && !T.ok(child)) child = -1;
    const bool visited = child != -1;
    const int safe = visited ? child : 0;
    depth += 1;
    load_row(safe);  // the next level's row when the walk goes on
    const bool selectable = row_outcome == kNoOutcome && searchable();
    cont = visited && selectable && depth < max_depth;
    next = child;
    k = next_key;
  }
  if (a == 0) {
    out_parent[b] = node;
    out_action[b] = action;
    out_active[b] = root_active;
  }
  if (stats) {
    const int pg = cta_reduce_add<W>(c, prior_gathers);
    if (a == 0) {
      atomicAdd(stats + 0, visited_nodes);
      atomicAdd(stats + 1, (unsigned long long)pg);
    }
  }
  if (parent_emb) {
    const int p = root_active ? node : 0;
    const uint8_t *src = T.embedding + T.node(b, p) * T.E;
    for (int i = a; i < T.E; i += 32 * W) parent_emb[(size_t)b * T.E + i] = src[i];
  }
}

// backward (search.py:146-171) with the built-in rules, one CTA per lane.
// RULE is the update rule of the launch (0: Monte Carlo, 1: guarded
// prefix-CDF).  With 2 matrices of [max(Q, 24)][96] floats and the shared
// Gamma-constant / zero-flag region, a 3-warp CTA takes 24.7 KB of shared
// memory at Q = 21 (24.0 KB for the Monte Carlo instance).  The register
// budgets are measured choices, not occupancy maxima: under a budget for
// 8 or 9 CTAs the prefix-CDF instance compiles to 10-16 % more
// instructions and, with more warps at different points of its large
// code, stalls more on instruction fetch, so it runs slower than under the
// budget for 6 (80 registers, 8 CTAs resident).  The Monte Carlo instance
// is fastest under the budget for 9.  The 4-warp instances keep budgets
// for 5 and 8, since tighter ones spill.
#ifndef SCACCHI_BWD_MIN_BLOCKS
#define SCACCHI_BWD_MIN_BLOCKS 6
#endif
#ifndef SCACCHI_BWD_MC_MIN_BLOCKS
#define SCACCHI_BWD_MC_MIN_BLOCKS 9
#endif

template <int W, int RULE>
__global__ void __launch_bounds__(32 * W, RULE == 1 ? (W < 4 ? SCACCHI_BWD_MIN_BLOCKS : 5)
                                                    : (W < 4 ? SCACCHI_BWD_MC_MIN_BLOCKS : 8))
    backward_cta_kernel(Tree T, const uint32_t *key, const int32_t *sim_parent, const int32_t *sim_action,
                        const uint8_t *sim_active, const float2 *step_value, const int32_t *step_tp, UpdateParams P,
                        unsigned long long *stats) {
  const int b = blockIdx.x, a = threadIdx.x;
  const Cta<W> c = cta_scratch<W>(RULE == 1 ? 2 * P.prefix.h + 1 : 1);
  const int A = T.A;
  const bool present = a < A;
  bool active = sim_active[b] != 0;
  int node = active ? sim_parent[b] : 0;
  if (!T.ok(node)) return;
  bool leaf_active = active;
  sk_key k = {key[0], key[1]};
  const int leaf_action_raw = sim_action[b];
  const int leaf_action = leaf_action_raw < 0 ? leaf_action_raw + A : leaf_action_raw;
  const float2 leaf_value = step_value[b];
  const int leaf_tp = step_tp[b];
  unsigned long long unsafe_n = 0, nodes = 0, child_gathers = 0;
  for (int level = 0; active && level < T.C; ++level) {
    const sk_key next_key = sk_split(k, 0), update_key = sk_split(k, 1);
    const size_t ni = T.node(b, node);
    const int node_tp = T.to_play[ni];
    const int node_payload = T.node_payload[ni];
    const float2 vprior = T.value_prior[ni], valpha = T.value_alpha[ni];
    const int8_t node_outcome = T.node_outcome[ni];
    // gather this thread's action (utils.py:35-50)
    float2 ea = make_float2(1.0f, 1.0f);
    int ep = 0;
    int8_t eo = kNoOutcome;
    bool inv = true, cvis = false;
    float2 cprior = ea, cvalue = ea;
    int cpay = 0, ctp = 0;
    int8_t cout = kNoOutcome;
    size_t e = 0;
    if (present) {
      e = T.edge(b, node, a);
      ea = T.edge_alpha[e];
      ep = T.edge_payload[e];
      eo = T.edge_outcome[e];
      inv = T.invalid[e] != 0;
      int child = T.children[e];
      cvis = child != -1;
      if (child != -1 && !T.ok(child)) child = -1;
      const size_t ci = T.node(b, child != -1 ? child : 0);
      cprior = T.value_prior[ci];
      cvalue = T.value_alpha[ci];
      cpay = T.node_payload[ci];
      cout = T.node_outcome[ci];
      ctp = T.to_play[ci];
    }
    // _repair_inputs, posterior_updates.py:66-190
    const bool unresolved = eo == kNoOutcome;
    float e0 = ea.x, e1 = ea.y;
    int nep = ep;
    if (leaf_active && a == leaf_action && unresolved) {
      const float2 d = align2(leaf_value, leaf_tp, node_tp);
      e0 = d.x;
      e1 = d.y;
      nep = nep + 1;
    }
    if (cvis && cout == kNoOutcome && cpay > 0 && unresolved) {
      const float2 cv = align2(cvalue, ctp, node_tp);
      e0 = cv.x;
      e1 = cv.y;
      nep = 1 + cpay;
    }
    float eff0 = e0, eff1 = e1;
    if (cvis && unresolved && nep <= 0) {
      const float2 cp = align2(cprior, ctp, node_tp);
      eff0 = cp.x;
      eff1 = cp.y;
    }
    float cache0 = eff0, cache1 = eff1;
    if (!unresolved) {
      const float s = eff0 + eff1;
      cache0 = s * (eo == 0 ? 1.0f : 0.0f);
      cache1 = s * (eo == 1 ? 1.0f : 0.0f);
    }
    const bool legal = present && !inv, unres = legal && unresolved;
    float amin = SM_INF;
    if (unres) {
      const float v0 = eff0 > SM_TINY ? eff0 : SM_TINY;
      const float v1 = eff1 > SM_TINY ? eff1 : SM_TINY;
      amin = v0 < v1 ? v0 : v1;
    }
    const NodeSummary sum = cta_node_summary<W>(c, legal, unres, legal && eo == 1, legal && eo == 0,
                                                unres ? nep - ep : 0, ep, amin, present && cvis);
    const int n_down = node_payload + sum.delta;
    // search policy: guarded prefix-CDF or Monte Carlo
    float policy = 0.0f;
    bool unsafe = false;
    if (RULE == 1) {
      const PrefixResult1 pr = cta_prefix_guarded<W>(c, sum, eff0, eff1, inv, eo, A, P.prefix, P.density_tol);
      policy = pr.policy;
      unsafe = pr.unsafe;
    }
    if (RULE != 1 || unsafe)
      policy = cta_mc_policy<W, RULE == 1 ? 1 : 2>(c, sum, update_key, eff0, eff1, inv, eo, P.samples, A, b, T.B);
    // mix_value_prior, posterior_updates.py:40-63
    float in2[2] = {policy * cache0, policy * cache1}, w2[2];
    cta_sums<W, 2>(c, in2, w2, A);
    const float n = (float)n_down;
    float pw, dw;
    if (P.kappa_ge_one) {
      const float rc = n * P.inv_kappa;
      const float den = 1.0f + rc;
      pw = 1.0f / den;
      dw = rc / den;
    } else {
      const float den = P.kappa + n;
      pw = P.kappa / den;
      dw = n / den;
    }
    const float2 repaired = make_float2(pw * vprior.x + dw * w2[0], pw * vprior.y + dw * w2[1]);
    const float2 new_value = n_down > 0 ? repaired : valpha;
    // _set_node_update (utils.py:53-64)
    if (present && unresolved) {
      T.edge_payload[e] = nep;
      T.edge_alpha[e] = make_float2(e0, e1);
    }
    // _categorize_node_and_publish (utils.py:67-124), binary outcomes
    const bool has_legal = sum.has_legal;
    const bool any_open = sum.n_unres > 0;
    const bool has_win = sum.has_win;
    const int shortest_win = sum.shortest_win;
    const int longest_loss = sum.longest_loss;
    const bool all_cat = has_legal && !any_open;
    const int8_t candidate = has_win ? 1 : (all_cat ? 0 : kNoOutcome);
    const int cdist = has_win ? shortest_win : longest_loss;
    const bool publish_node = node_outcome == kNoOutcome && candidate != kNoOutcome;
    int sp = 0, ia = 0;
    bool has_parent = false, has_incoming = false;
    if (publish_node) {
      const int parent = T.parents[ni];
      has_parent = parent != -1 && T.ok(parent);
      sp = has_parent ? parent : 0;
      const int first =
          cta_reduce_min<W>(c, (present && T.children[T.edge(b, sp, a)] == node) ? a : INT_MAX);
      has_incoming = first != INT_MAX;
      ia = has_incoming ? first : 0;
    }
    if (a == 0) {
      T.node_payload[ni] = n_down;
      T.value_alpha[ni] = new_value;
      if (publish_node) {
        const size_t pe = T.edge(b, sp, ia), pn = T.node(b, sp);
        const bool publish_edge = has_parent && has_incoming && T.edge_outcome[pe] == kNoOutcome;
        const int new_support = T.node_payload[pn] + 1 + n_down - T.edge_payload[pe];
        const int8_t aligned = align_cat(candidate, node_tp, T.to_play[pn]);
        if (publish_edge) T.node_payload[pn] = new_support;
        T.node_payload[ni] = cdist;
        T.node_outcome[ni] = candidate;
        if (publish_edge) {
          T.edge_outcome[pe] = aligned;
          T.edge_payload[pe] = cdist + 1;
        }
      }
    }
    unsafe_n += unsafe;
    nodes += 1;
    child_gathers += (unsigned long long)sum.visited;
    __syncthreads();
    const bool up = node != 0;
    const int parent = T.parents[ni];
    if (up && !T.ok(parent)) break;
    node = up ? parent : 0;
    active = up;
    leaf_active = false;
    k = next_key;
  }
  if (stats && a == 0) {
    atomicAdd(stats + 0, nodes);
    atomicAdd(stats + 1, child_gathers);
    if (unsafe_n) atomicAdd(stats + 2, unsafe_n);
  }
}
