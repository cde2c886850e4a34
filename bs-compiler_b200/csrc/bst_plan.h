// bst_plan.h — work plans of the persistent march kernels (host only).
//
// choose_chunks: equal items (tile column x M-chunk) that fill whole waves of resident CTAs.
// choose_item_plan: the same, or a two-band plan whose finer second band fills the last wave.
#pragma once

#include <algorithm>
#include <functional>
#include <mutex>
#include <unordered_map>
#include <utility>
#include <vector>

namespace bst {

// Choose the M-chunk so that equal-size items fill whole waves of resident CTAs.  The scan
// covers up to 4096 chunk counts, so results are remembered per request shape (a multi-pass
// run repeats the same few shapes, and the host must enqueue a pass faster than it runs).
inline void choose_chunks_scan(long long base_tiles, long long nm, int rb, int overhead, long long resident,
                               int* chunk_out, long long* nchunks_out);
inline void choose_chunks(long long base_tiles, long long nm, int rb, int overhead, long long resident,
                          int* chunk_out, long long* nchunks_out) {
  struct Key {
    long long t, m, res;
    int rb, ov;
    bool operator==(const Key& o) const { return t == o.t && m == o.m && res == o.res && rb == o.rb && ov == o.ov; }
  };
  struct KeyHash {
    size_t operator()(const Key& k) const {
      return std::hash<long long>()(k.t * 1000003LL ^ k.m * 7919LL ^ k.res) ^ (size_t(k.rb) << 20) ^ size_t(k.ov);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, std::pair<int, long long>, KeyHash> memo;
  const Key key{base_tiles, nm, resident, rb, overhead};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = memo.find(key);
    if (it != memo.end()) {
      *chunk_out = it->second.first;
      *nchunks_out = it->second.second;
      return;
    }
  }
  choose_chunks_scan(base_tiles, nm, rb, overhead, resident, chunk_out, nchunks_out);
  std::lock_guard<std::mutex> lk(mu);
  if (memo.size() > 4096) memo.clear();
  memo.emplace(key, std::make_pair(*chunk_out, *nchunks_out));
}

inline void choose_chunks_scan(long long base_tiles, long long nm, int rb, int overhead, long long resident,
                               int* chunk_out, long long* nchunks_out) {
  double best = 1e300;
  int best_chunk = int(nm);
  long long best_n = 1;
  const long long max_nc = nm / rb + 1;
  for (long long nc = 1; nc <= max_nc && nc <= 4096; ++nc) {
    long long chunk = (nm + nc - 1) / nc;
    chunk = (chunk + rb - 1) / rb * rb;
    const long long real = (nm + chunk - 1) / chunk;
    const long long items = base_tiles * real;
    const long long waves = (items + resident - 1) / resident;
    const double t = double(waves) * double(chunk + overhead);
    if (t < best * 0.999) {
      best = t;
      best_chunk = int(chunk);
      best_n = real;
    }
  }
  *chunk_out = best_chunk;
  *nchunks_out = best_n;
}

// Two-band item plan.  Equal items on a persistent grid of S CTAs (CTA b takes items b, b+S,
// ...) quantise into whole waves: 1024 tile columns on 296 resident CTAs fill 3.46 waves, and
// cutting every column into more chunks pays the Z-window ramp once more per chunk.  Cutting
// only some columns one chunk finer, and listing those smaller items last, fills the last
// wave instead.  A model of the launch (an item costs its planes plus a fixed ramp; CTAs take
// items round-robin) scores the uniform plan and the two-band ones; the cheapest wins, the
// uniform plan unless a split saves more than 1 %.  Results are remembered per shape.
struct ItemPlan {
  long long tiles1 = 0, n1 = 0, n2 = 0;
  int chunk1 = 0, chunk2 = 0;
};

inline long long plan_cost(const ItemPlan& p, long long tiles, long long nm, int overhead, long long S,
                           std::vector<long long>& loads) {
  loads.assign(size_t(S), 0);
  long long w = 0;
  auto band = [&](long long ntiles, long long n, long long ch) {
    for (long long ci = 0; ci < n; ++ci) {
      const long long size = std::min(ch, nm - ci * ch) + overhead;
      for (long long t = 0; t < ntiles; ++t, ++w) loads[size_t(w % S)] += size;
    }
  };
  band(p.tiles1, p.n1, p.chunk1);
  band(tiles - p.tiles1, p.n2, p.chunk2);
  return *std::max_element(loads.begin(), loads.end());
}

inline ItemPlan choose_item_plan(long long tiles, long long nm, int rb, int overhead, long long resident) {
  struct Key {
    long long t, m, res;
    int rb, ov;
    bool operator==(const Key& o) const { return t == o.t && m == o.m && res == o.res && rb == o.rb && ov == o.ov; }
  };
  struct KeyHash {
    size_t operator()(const Key& k) const {
      return std::hash<long long>()(k.t * 1000003LL ^ k.m * 7919LL ^ k.res) ^ (size_t(k.rb) << 20) ^ size_t(k.ov);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, ItemPlan, KeyHash> memo;
  const Key key{tiles, nm, resident, rb, overhead};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
  }
  auto split = [&](long long n, int* ch, long long* real) {  // n chunks of whole RB groups
    long long c = (nm + n - 1) / n;
    c = (c + rb - 1) / rb * rb;
    *ch = int(c);
    *real = (nm + c - 1) / c;
  };
  int chunk = 0;
  long long nchunks = 1;
  choose_chunks(tiles, nm, rb, overhead, resident, &chunk, &nchunks);
  ItemPlan best;
  best.tiles1 = tiles;
  best.chunk1 = best.chunk2 = chunk;
  best.n1 = best.n2 = nchunks;
  const long long S = resident > 0 ? resident : 1;
  std::vector<long long> loads;
  const long long uniform = plan_cost(best, tiles, nm, overhead, S, loads);
  long long best_cost = uniform;
  if (tiles >= 2 && tiles * (nchunks + 1) > S && tiles * nchunks * 4 <= 65536) {
    const long long step = std::max<long long>(1, tiles / 64);
    for (long long n = 1; n <= 4 && n * rb <= nm; ++n) {
      ItemPlan p;
      long long r1 = 0, r2 = 0;
      split(n, &p.chunk1, &r1);
      split(n + 1, &p.chunk2, &r2);
      if (r2 <= r1) continue;  // the finer band must really be finer
      p.n1 = r1;
      p.n2 = r2;
      for (long long t1 = step; t1 < tiles; t1 += step) {
        p.tiles1 = t1;
        const long long cost = plan_cost(p, tiles, nm, overhead, S, loads);
        if (cost < best_cost) {
          best_cost = cost;
          best = p;
        }
      }
    }
    if (best_cost * 100 > uniform * 99) {  // under 1 %: keep the uniform plan
      best.tiles1 = tiles;
      best.chunk1 = best.chunk2 = chunk;
      best.n1 = best.n2 = nchunks;
    }
  }
  std::lock_guard<std::mutex> lk(mu);
  if (memo.size() > 4096) memo.clear();
  memo.emplace(key, best);
  return best;
}

}  // namespace bst
