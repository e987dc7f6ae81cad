// Hex on the GPU: the environment step, observation and legal mask the
// search's recurrent function needs (scacchi/envs.py:98-125 wraps pgx
// 2.6.0's Hex; dirichlet_q_search.py:43-76 turns a step into the search's
// RecurrentFnOutput), plus the seeded root sampler of the full-step
// workload.
//
// A lane's state is a 48-byte record holding two bitboards (black, white;
// bit r * size + c) and a few bytes of turn state, so the tree stores a
// whole game state per node in 48 bytes.  One warp serves one lane: every
// thread computes the step on the bitboards (a few hundred integer
// operations, identical in all threads), then the warp writes the
// observation, legal row and outputs with coalesced strided stores.
//
// Rules: black (colour 0) moves first and connects row 0 to row size-1,
// white connects column 0 to column size-1; neighbours of (r, c) are
// (r-1, c), (r-1, c+1), (r, c-1), (r, c+1), (r+1, c-1), (r+1, c).  The swap
// action (index size * size) is never legal (envs.py:107,117); at a terminal
// state every action reads legal, pgx's convention.

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/scacchi_b200.h"
#include "threefry.h"

namespace {

constexpr int kHexMaxSize = 11;  // 121 cells fit two 64-bit words
constexpr int kHexWarpsPerBlock = 4;
std::atomic<uint64_t> g_hex_launches{0};

struct __align__(16) HexRecord {
  uint64_t black[2];
  uint64_t white[2];
  uint8_t color;         // colour to move: 0 black, 1 white
  uint8_t black_player;  // player id playing black (player_order[0])
  uint8_t terminated;
  int8_t winner;         // colour that connected, -1 none
  uint8_t size;
  uint8_t moves;         // stones placed
  uint8_t pad[10];
};
static_assert(sizeof(HexRecord) == SCACCHI_HEX_RECORD_BYTES, "record layout");

struct Bits {
  uint64_t lo, hi;
};

__device__ __forceinline__ Bits b_or(Bits a, Bits b) { return {a.lo | b.lo, a.hi | b.hi}; }
__device__ __forceinline__ Bits b_and(Bits a, Bits b) { return {a.lo & b.lo, a.hi & b.hi}; }
__device__ __forceinline__ Bits b_andnot(Bits a, Bits b) { return {a.lo & ~b.lo, a.hi & ~b.hi}; }
__device__ __forceinline__ bool b_any(Bits a) { return (a.lo | a.hi) != 0; }
__device__ __forceinline__ bool b_eq(Bits a, Bits b) { return a.lo == b.lo && a.hi == b.hi; }
__device__ __forceinline__ int b_popc(Bits a) { return __popcll(a.lo) + __popcll(a.hi); }
__device__ __forceinline__ bool b_test(Bits a, int i) { return ((i < 64 ? a.lo >> i : a.hi >> (i - 64)) & 1) != 0; }
__device__ __forceinline__ Bits b_bit(int i) {
  return i < 64 ? Bits{1ull << i, 0} : Bits{0, 1ull << (i - 64)};
}
// shifts by 1 <= n <= 63
__device__ __forceinline__ Bits b_shl(Bits a, int n) { return {a.lo << n, (a.hi << n) | (a.lo >> (64 - n))}; }
__device__ __forceinline__ Bits b_shr(Bits a, int n) { return {(a.lo >> n) | (a.hi << (64 - n)), a.hi >> n}; }

struct Masks {
  Bits board, col_first, col_last, row_first, row_last;
};

__device__ Masks make_masks(int s) {
  Masks m{{0, 0}, {0, 0}, {0, 0}, {0, 0}, {0, 0}};
  for (int r = 0; r < s; ++r)
    for (int c = 0; c < s; ++c) {
      const Bits bit = b_bit(r * s + c);
      m.board = b_or(m.board, bit);
      if (c == 0) m.col_first = b_or(m.col_first, bit);
      if (c == s - 1) m.col_last = b_or(m.col_last, bit);
      if (r == 0) m.row_first = b_or(m.row_first, bit);
      if (r == s - 1) m.row_last = b_or(m.row_last, bit);
    }
  return m;
}

// Cells of `own` joined to the colour's first edge, grown one neighbour ring
// at a time; true when the growth reaches the second edge.
__device__ bool connected(Bits own, int s, int colour, const Masks &m) {
  const Bits goal = colour == 0 ? m.row_last : m.col_last;
  Bits reach = b_and(own, colour == 0 ? m.row_first : m.col_first);
  for (int it = 0; it <= kHexMaxSize * kHexMaxSize; ++it) {
    if (b_any(b_and(reach, goal))) return true;
    const Bits not_last = b_andnot(reach, m.col_last), not_first = b_andnot(reach, m.col_first);
    Bits nb = reach;
    nb = b_or(nb, b_shr(reach, s));               // (r-1, c)
    nb = b_or(nb, b_shr(not_last, s - 1));        // (r-1, c+1)
    nb = b_or(nb, b_shr(not_first, 1));           // (r, c-1)
    nb = b_or(nb, b_shl(not_last, 1));            // (r, c+1)
    nb = b_or(nb, b_shl(not_first, s - 1));       // (r+1, c-1)
    nb = b_or(nb, b_shl(reach, s));               // (r+1, c)
    const Bits next = b_and(nb, own);
    if (b_eq(next, reach)) return false;
    reach = next;
  }
  return b_any(b_and(reach, goal));
}

__device__ __forceinline__ Bits stones(const uint64_t *w) { return {w[0], w[1]}; }

__device__ __forceinline__ int current_player(const HexRecord &h) {
  return h.color == 0 ? h.black_player : 1 - h.black_player;
}

// Place the mover's stone on `cell` (empty, state not terminal).
__device__ HexRecord place(HexRecord h, int cell, const Masks &m) {
  const int s = h.size;
  const Bits bit = b_bit(cell);
  Bits own;
  if (h.color == 0) {
    own = b_or(stones(h.black), bit);
    h.black[0] = own.lo;
    h.black[1] = own.hi;
  } else {
    own = b_or(stones(h.white), bit);
    h.white[0] = own.lo;
    h.white[1] = own.hi;
  }
  h.moves += 1;
  if (connected(own, s, h.color, m)) {
    h.terminated = 1;
    h.winner = (int8_t)h.color;
  }
  h.color = 1 - h.color;
  return h;
}

// A record viewed as the 16-byte words it is moved in.
union RecordWords {
  HexRecord h;
  uint4 v[3];
  uint32_t w[12];
};
static_assert(sizeof(RecordWords) == sizeof(HexRecord), "record words");

__device__ __forceinline__ HexRecord load_record(const uint8_t *p) {
  const uint4 *src = reinterpret_cast<const uint4 *>(p);
  RecordWords u;
  u.v[0] = src[0];
  u.v[1] = src[1];
  u.v[2] = src[2];
  return u.h;
}

// Warp-cooperative writes of one lane's derived outputs.
struct Outputs {
  float *observation;       // [B, s, s, 4]
  uint8_t *invalid;         // [B, s*s + 1]
  int8_t *terminal;         // [B] terminal outcome aligned to the state's player (or -1)
  int32_t *to_play;         // [B]
  float *rewards;           // [B, 2]
  uint8_t *terminated;      // [B]
};

__device__ void write_outputs(const HexRecord &h, int b, int lane, const Outputs &o, int parent_player) {
  const int s = h.size, cells = s * s, A = cells + 1;
  const Bits black = stones(h.black), white = stones(h.white);
  const Bits own = h.color == 0 ? black : white, opp = h.color == 0 ? white : black;
  if (o.observation) {
    float *obs = o.observation + (size_t)b * cells * 4;
    const float colour_plane = (float)h.color, second_move = h.moves == 1 ? 1.0f : 0.0f;
    for (int i = lane; i < cells * 4; i += 32) {
      const int cell = i >> 2, plane = i & 3;
      float v;
      if (plane == 0) v = b_test(own, cell) ? 1.0f : 0.0f;
      else if (plane == 1) v = b_test(opp, cell) ? 1.0f : 0.0f;
      else if (plane == 2) v = colour_plane;
      else v = second_move;
      obs[i] = v;
    }
  }
  if (o.invalid) {
    uint8_t *inv = o.invalid + (size_t)b * A;
    const Bits filled = b_or(black, white);
    for (int a = lane; a < A; a += 32) {
      const bool legal = h.terminated ? true : (a < cells && !b_test(filled, a));
      inv[a] = legal ? 0 : 1;
    }
  }
  if (lane == 0) {
    const int player = current_player(h);
    float r_win = 0.0f, r_lose = 0.0f;
    int win_player = -1;
    if (h.terminated) {
      win_player = h.winner == 0 ? h.black_player : 1 - h.black_player;
      r_win = 1.0f;
      r_lose = -1.0f;
    }
    if (o.rewards) {
      o.rewards[2 * b + 0] = win_player < 0 ? 0.0f : (win_player == 0 ? r_win : r_lose);
      o.rewards[2 * b + 1] = win_player < 0 ? 0.0f : (win_player == 1 ? r_win : r_lose);
    }
    if (o.terminated) o.terminated[b] = h.terminated;
    if (o.to_play) o.to_play[b] = player;
    if (o.terminal) {
      // dirichlet_q_search.py:53-66: the reward of the parent's player gives
      // the parent-perspective outcome (round(r) + 1) / 2, aligned to the
      // player to move here; -1 for a non-terminal state.  Without a parent
      // the state's own player is the reference.
      int8_t t = -1;
      if (h.terminated) {
        const int ref = parent_player < 0 ? player : parent_player;
        const int outcome = (ref == win_player) ? 1 : 0;
        t = (int8_t)(ref == player ? outcome : 1 - outcome);
      }
      o.terminal[b] = t;
    }
  }
}

__device__ __forceinline__ void store_record(uint8_t *dst, const HexRecord &h, int lane) {
  RecordWords u;
  u.h = h;
  if (lane < 12) reinterpret_cast<uint32_t *>(dst)[lane] = u.w[lane];
}

__global__ void __launch_bounds__(32 * kHexWarpsPerBlock)
    hex_step_kernel(int B, const uint8_t *states, const int32_t *action, uint8_t *next_states, Outputs o,
                    uint32_t *error) {
  const int b = blockIdx.x * kHexWarpsPerBlock + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b >= B) return;
  const HexRecord h = load_record(states + (size_t)b * sizeof(HexRecord));
  const int s = h.size;
  HexRecord n = h;
  const int a = action[b];
  const bool bad_size = s < 2 || s > kHexMaxSize;
  const int cells = bad_size ? 0 : s * s;
  bool ok = !bad_size && !h.terminated && a >= 0 && a < cells;
  if (ok) {
    const Bits filled = b_or(stones(h.black), stones(h.white));
    ok = !b_test(filled, a);
  }
  // An illegal action or a terminal parent returns the state unchanged: the
  // search steps every lane and passes action 0 for lanes with nothing to
  // expand, whose results it discards.
  if (ok) {
    const Masks m = make_masks(s);
    n = place(h, a, m);
  }
  if (bad_size) {
    if (lane == 0) atomicOr(error, 1u);
    return;
  }
  store_record(next_states + (size_t)b * sizeof(HexRecord), n, lane);
  write_outputs(n, b, lane, o, current_player(h));
}

__global__ void __launch_bounds__(32 * kHexWarpsPerBlock)
    hex_observe_kernel(int B, const uint8_t *states, Outputs o, uint32_t *error) {
  const int b = blockIdx.x * kHexWarpsPerBlock + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b >= B) return;
  const HexRecord h = load_record(states + (size_t)b * sizeof(HexRecord));
  if (h.size < 2 || h.size > kHexMaxSize) {
    if (lane == 0) atomicOr(error, 1u);
    return;
  }
  write_outputs(h, b, lane, o, -1);
}

__device__ HexRecord empty_record(int s, int black_player) {
  HexRecord h;
  h.black[0] = h.black[1] = h.white[0] = h.white[1] = 0;
  h.color = 0;
  h.black_player = (uint8_t)black_player;
  h.terminated = 0;
  h.winner = -1;
  h.size = (uint8_t)s;
  h.moves = 0;
  for (int i = 0; i < 10; ++i) h.pad[i] = 0;
  return h;
}

// envs.py:103-112: player_order = [[0, 1], [1, 0]][bernoulli(key)], so the
// player playing black is 1 when uniform(key) < 0.5.
__device__ __forceinline__ int black_player_of(sk_key k) { return sk_uniform(k, 0, 0.0f, 1.0f) < 0.5f ? 1 : 0; }

__global__ void __launch_bounds__(32 * kHexWarpsPerBlock)
    hex_init_kernel(int B, int s, const uint32_t *keys, uint8_t *states) {
  const int b = blockIdx.x * kHexWarpsPerBlock + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b >= B) return;
  const sk_key k = {keys[2 * b], keys[2 * b + 1]};
  store_record(states + (size_t)b * sizeof(HexRecord), empty_record(s, black_player_of(k)), lane);
}

// Seeded roots: lane key k = fold_in(key, lane); player order from
// bernoulli(fold_in(k, 0)); min_moves + bits(fold_in(k, 1)) % span random
// legal moves, move j taking the (bits(fold_in(k, 2 + j)) % n)-th empty
// cell in index order; a terminal state ends the sequence.
__global__ void __launch_bounds__(32 * kHexWarpsPerBlock)
    hex_random_roots_kernel(int B, int s, sk_key key, int min_moves, int span, uint8_t *states) {
  const int b = blockIdx.x * kHexWarpsPerBlock + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b >= B) return;
  const sk_key k = sk_fold_in(key, (uint32_t)b);
  HexRecord h = empty_record(s, black_player_of(sk_fold_in(k, 0)));
  const int n = min_moves + (int)(sk_bits(sk_fold_in(k, 1), 0) % (uint32_t)span);
  const Masks m = make_masks(s);
  for (int j = 0; j < n && !h.terminated; ++j) {
    const Bits empty = b_andnot(m.board, b_or(stones(h.black), stones(h.white)));
    const int count = b_popc(empty);
    if (count == 0) break;
    int pick = (int)(sk_bits(sk_fold_in(k, 2u + (uint32_t)j), 0) % (uint32_t)count);
    int cell = -1;
    for (int i = 0; i < s * s; ++i) {
      if (b_test(empty, i)) {
        if (pick == 0) {
          cell = i;
          break;
        }
        --pick;
      }
    }
    if (cell < 0) break;
    h = place(h, cell, m);
  }
  store_record(states + (size_t)b * sizeof(HexRecord), h, lane);
}

__device__ uint32_t g_hex_error;

int hex_blocks(int B) { return (B + kHexWarpsPerBlock - 1) / kHexWarpsPerBlock; }

int hex_launched() {
  g_hex_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError() == cudaSuccess ? SCACCHI_OK : SCACCHI_ECUDA;
}

}  // namespace

extern "C" {

int scacchi_hex_init(int32_t batch, int32_t size, const uint32_t *keys, uint8_t *states, void *stream) {
  if (batch < 0 || size < 2 || size > kHexMaxSize || (batch > 0 && (!keys || !states))) return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  hex_init_kernel<<<hex_blocks(batch), 32 * kHexWarpsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      batch, size, keys, states);
  return hex_launched();
}

int scacchi_hex_random_roots(int32_t batch, int32_t size, uint32_t key0, uint32_t key1, int32_t min_moves,
                             int32_t max_moves, uint8_t *states, void *stream) {
  if (batch < 0 || size < 2 || size > kHexMaxSize || min_moves < 0 || max_moves < min_moves ||
      max_moves > size * size || (batch > 0 && !states))
    return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  hex_random_roots_kernel<<<hex_blocks(batch), 32 * kHexWarpsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      batch, size, sk_key{key0, key1}, min_moves, max_moves - min_moves + 1, states);
  return hex_launched();
}

int scacchi_hex_step(int32_t batch, const uint8_t *states, const int32_t *action, uint8_t *next_states,
                     float *observation, uint8_t *invalid, int8_t *terminal_outcome, int32_t *to_play,
                     float *rewards, uint8_t *terminated, void *stream) {
  if (batch < 0 || (batch > 0 && (!states || !action || !next_states))) return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  uint32_t *err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_hex_error) != cudaSuccess) return SCACCHI_ECUDA;
  const Outputs o{observation, invalid, terminal_outcome, to_play, rewards, terminated};
  hex_step_kernel<<<hex_blocks(batch), 32 * kHexWarpsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      batch, states, action, next_states, o, err);
  return hex_launched();
}

int scacchi_hex_observe(int32_t batch, const uint8_t *states, float *observation, uint8_t *invalid,
                        int8_t *terminal_outcome, int32_t *to_play, float *rewards, uint8_t *terminated,
                        void *stream) {
  if (batch < 0 || (batch > 0 && !states)) return SCACCHI_EINVAL;
  if (batch == 0) return SCACCHI_OK;
  uint32_t *err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_hex_error) != cudaSuccess) return SCACCHI_ECUDA;
  const Outputs o{observation, invalid, terminal_outcome, to_play, rewards, terminated};
  hex_observe_kernel<<<hex_blocks(batch), 32 * kHexWarpsPerBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      batch, states, o, err);
  return hex_launched();
}

int scacchi_hex_error(uint32_t *flags) {
  if (!flags) return SCACCHI_EINVAL;
  uint32_t v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_hex_error, sizeof(v)) != cudaSuccess) return SCACCHI_ECUDA;
  if (cudaMemcpyToSymbol(g_hex_error, &zero, sizeof(zero)) != cudaSuccess) return SCACCHI_ECUDA;
  *flags = v;
  return SCACCHI_OK;
}

uint64_t scacchi_hex_launch_count(void) { return g_hex_launches.load(std::memory_order_relaxed); }

}  // extern "C"
