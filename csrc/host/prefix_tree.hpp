// Radix prefix cache over full KV pages (reference semantics of
// prefix/radix/index.mbt:11-406 and eviction.mbt:2): trees rooted per prefix
// identity, only full pages stored or returned, per-node active references,
// least-recently-used eviction of unreferenced leaves, and a *cached*
// reference held on every stored page through the page allocator.
//
// Layout: nodes live in a slot vector (freed slots are reused; a per-slot
// epoch invalidates stale heap entries).  Each edge is one page of tokens,
// kept in a flat token array (P int32 per node).  A child is found through
// one hash map keyed by (parent slot, 64-bit hash of the page's tokens); the
// tokens are compared on a hit, and colliding siblings chain through
// `next_same`.  A lookup is O(pages); eviction pops (recency, push order)
// from a min-heap.  The recency clock, the push order and the stale-entry
// rules are those of the Python reference class PrefixIndex
// (lunaflux_b200/prefix/radix.py), so both evict in the same order; the
// tests run them side by side.
#pragma once
#include <cstdint>
#include <cstring>
#include <queue>
#include <stdexcept>
#include <tuple>
#include <unordered_map>
#include <utility>
#include <vector>

#include "page_allocator.hpp"

namespace lf_host {

class PrefixError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

class PrefixTree {
 public:
  using Page = std::pair<int, int64_t>;

  PrefixTree(PageAllocator& alloc, int tokens_per_page, int64_t max_pages)
      : alloc_(alloc), P_(tokens_per_page), max_pages_(max_pages) {
    if (tokens_per_page <= 0) throw PrefixError("tokens_per_page must be positive");
  }

  int tokens_per_page() const { return P_; }

  int new_root() {
    const int n = make_node(-1, nullptr, {0, 0}, 0);
    nodes_[n].root = true;
    ++roots_;
    return n;
  }

  // Longest chain of cached full pages prefixing tokens[0:n] (at most
  // max_pages pages; negative: no limit).  Returns node slots, root excluded.
  std::vector<int> lookup(int root, const int32_t* toks, int64_t n, int64_t max_pages) {
    return lookup_with(root, n, max_pages, [toks, this](int64_t i) { return toks + i * P_; });
  }

  // The same walk over a token source: page_of(i) returns page i's P tokens
  // (valid until the next call).  Pages past the first mismatch are never read.
  template <class PageOf>
  std::vector<int> lookup_with(int root, int64_t n, int64_t max_pages, PageOf&& page_of) {
    check_root(root);
    ++lookups_;
    int64_t n_full = n / P_;
    if (max_pages >= 0 && max_pages < n_full) n_full = max_pages;
    const int64_t now = ++clock_;
    std::vector<int> out;
    int node = root;
    for (int64_t i = 0; i < n_full; ++i) {
      if (nodes_[node].nchildren == 0) break;
      const int c = find_child(node, page_of(i));
      if (c < 0) break;
      nodes_[c].recency = now;
      out.push_back(c);
      node = c;
    }
    if (!out.empty()) {
      ++hits_;
      hit_tokens_ += (int64_t)out.size() * P_;
      push_leaf(out.back());
    }
    return out;
  }

  void retain(const std::vector<int>& ns) {
    for (int n : ns) ++live(n).refs;
  }

  void release(const std::vector<int>& ns) {
    for (int n : ns) {
      Node& x = live(n);
      if (x.refs <= 0) throw PrefixError("prefix node released more often than retained");
      if (--x.refs == 0 && x.nchildren == 0) push_leaf(n);
    }
  }

  // Publishes the full pages of tokens[0:n] (pages[i] holds page i's KV).
  // Returns the pages newly cached.
  int insert(int root, const int32_t* toks, int64_t n, const std::vector<Page>& pages) {
    return insert_with(root, n, pages, [toks, this](int64_t i) { return toks + i * P_; });
  }

  template <class PageOf>
  int insert_with(int root, int64_t n, const std::vector<Page>& pages, PageOf&& page_of) {
    check_root(root);
    int64_t n_full = n / P_;
    if ((int64_t)pages.size() < n_full) n_full = (int64_t)pages.size();
    int added = 0;
    const int64_t now = ++clock_;
    int node = root;
    for (int64_t i = 0; i < n_full; ++i) {
      const int32_t* key = page_of(i);
      int c = find_child(node, key);
      if (c < 0) {
        if (count_ >= max_pages_) break;
        alloc_.retain_cached(pages[i].first, pages[i].second);
        c = make_node(node, key, pages[i], nodes_[node].depth + 1);
        link_child(node, c);
        ++count_;
        ++added;
      }
      nodes_[c].recency = now;
      node = c;
    }
    if (!nodes_[node].root && nodes_[node].nchildren == 0) push_leaf(node);
    return added;
  }

  // Evicts least-recently-used unreferenced leaves until `need` pages were
  // released or nothing evictable remains; returns the pages released.
  int evict(int64_t need) {
    int freed = 0;
    while (freed < need && !heap_.empty()) {
      const HeapEntry e = heap_.top();
      heap_.pop();
      const int n = e.node;
      if (epoch_[n] != e.epoch) continue;  // the slot was freed (and maybe reused) since the push
      Node& x = nodes_[n];
      if (x.root || x.nchildren > 0 || x.refs > 0 || e.recency != x.recency) {
        if (!x.root && x.nchildren == 0 && x.refs == 0 && e.recency != x.recency) push_leaf(n);
        continue;
      }
      const int parent = x.parent;
      unlink_child(parent, n);
      const Page pg = x.page;
      free_node(n);
      alloc_.release_cached(pg.first, pg.second);
      --count_;
      ++evicted_;
      ++freed;
      const Node& p = nodes_[parent];
      if (!p.root && p.nchildren == 0 && p.refs == 0) push_leaf(parent);
    }
    return freed;
  }

  Page page(int n) const { return live_c(n).page; }
  std::vector<Page> pages_of(const std::vector<int>& ns) const {
    std::vector<Page> out;
    out.reserve(ns.size());
    for (int n : ns) out.push_back(live_c(n).page);
    return out;
  }

  int64_t page_count() const { return count_; }
  int64_t evictable_pages() const {
    int64_t c = 0;
    for (size_t n = 0; n < nodes_.size(); ++n)
      if (nodes_[n].used && !nodes_[n].root && nodes_[n].refs == 0) ++c;
    return c;
  }
  int64_t hits() const { return hits_; }
  int64_t lookups() const { return lookups_; }
  int64_t hit_tokens() const { return hit_tokens_; }
  int64_t evicted_pages() const { return evicted_; }

  void debug_check_invariants() const {
    int64_t total = 0;
    std::vector<int> kids(nodes_.size(), 0);
    for (size_t n = 0; n < nodes_.size(); ++n) {
      const Node& x = nodes_[n];
      if (!x.used || x.root) continue;
      ++total;
      if (x.parent < 0 || !nodes_[x.parent].used) throw PrefixError("node without a live parent");
      if (x.depth != nodes_[x.parent].depth + 1) throw PrefixError("node depth");
      if (find_child(x.parent, key_of((int)n)) != (int)n) throw PrefixError("node not reachable from its parent");
      if (alloc_.cached_reference_count(x.page.first, x.page.second) < 1) throw PrefixError("stored page not cached");
      ++kids[x.parent];
    }
    for (size_t n = 0; n < nodes_.size(); ++n)
      if (nodes_[n].used && kids[n] != nodes_[n].nchildren) throw PrefixError("child count");
    if (total != count_) throw PrefixError("page count");
  }

 private:
  struct Node {
    int parent = -1;
    int nchildren = 0;
    int next_same = -1;  // next sibling with the same key hash
    int refs = 0;
    int depth = 0;
    bool root = false;
    bool used = false;
    uint64_t hash = 0;
    int64_t recency = 0;
    Page page{0, 0};
  };
  struct HeapEntry {
    int64_t recency;
    int64_t order;
    int node;
    uint32_t epoch;
    bool operator>(const HeapEntry& o) const {
      return std::tie(recency, order) > std::tie(o.recency, o.order);
    }
  };
  static uint64_t mix(uint64_t h) {
    h ^= h >> 33;
    h *= 0xff51afd7ed558ccdULL;
    h ^= h >> 33;
    return h;
  }
  uint64_t hash_page(const int32_t* k) const {
    uint64_t h = 0x9ae16a3b2f90404fULL;
    for (int i = 0; i < P_; ++i) h = mix(h ^ (uint32_t)k[i]) + 0x632be59bd9b4e019ULL;
    return h;
  }
  static uint64_t edge_key(int parent, uint64_t h) { return mix(h ^ ((uint64_t)(uint32_t)parent * 0x9e3779b97f4a7c15ULL)); }

  const int32_t* key_of(int n) const { return keys_.data() + (size_t)n * P_; }

  int find_child(int parent, const int32_t* key) const {
    if (nodes_[parent].nchildren == 0) return -1;
    const uint64_t h = hash_page(key);
    auto it = children_.find(edge_key(parent, h));
    for (int c = it == children_.end() ? -1 : it->second; c >= 0; c = nodes_[c].next_same)
      if (nodes_[c].parent == parent && nodes_[c].hash == h && std::memcmp(key_of(c), key, sizeof(int32_t) * P_) == 0)
        return c;
    return -1;
  }

  void link_child(int parent, int c) {
    auto [it, fresh] = children_.try_emplace(edge_key(parent, nodes_[c].hash), c);
    if (!fresh) {
      nodes_[c].next_same = it->second;
      it->second = c;
    }
    ++nodes_[parent].nchildren;
  }

  void unlink_child(int parent, int c) {
    const uint64_t ek = edge_key(parent, nodes_[c].hash);
    auto it = children_.find(ek);
    if (it == children_.end()) throw PrefixError("child edge missing");
    if (it->second == c) {
      if (nodes_[c].next_same >= 0)
        it->second = nodes_[c].next_same;
      else
        children_.erase(it);
    } else {
      int p = it->second;
      while (p >= 0 && nodes_[p].next_same != c) p = nodes_[p].next_same;
      if (p < 0) throw PrefixError("child edge missing");
      nodes_[p].next_same = nodes_[c].next_same;
    }
    --nodes_[parent].nchildren;
  }

  int make_node(int parent, const int32_t* key, Page page, int depth) {
    int n;
    if (!free_.empty()) {
      n = free_.back();
      free_.pop_back();
    } else {
      n = (int)nodes_.size();
      nodes_.emplace_back();
      epoch_.push_back(0);
      keys_.resize(keys_.size() + P_);
    }
    Node& x = nodes_[n];
    x = Node();
    x.used = true;
    x.parent = parent;
    x.page = page;
    x.depth = depth;
    if (key != nullptr) {
      std::memcpy(keys_.data() + (size_t)n * P_, key, sizeof(int32_t) * P_);
      x.hash = hash_page(key);
    }
    return n;
  }

  void free_node(int n) {
    nodes_[n].used = false;
    ++epoch_[n];
    free_.push_back(n);
  }

  void push_leaf(int n) { heap_.push({nodes_[n].recency, ++order_, n, epoch_[n]}); }

  void check_root(int r) const {
    if (r < 0 || r >= (int)nodes_.size() || !nodes_[r].used || !nodes_[r].root) throw PrefixError("unknown root");
  }
  Node& live(int n) {
    if (n < 0 || n >= (int)nodes_.size() || !nodes_[n].used || nodes_[n].root) throw PrefixError("stale prefix node");
    return nodes_[n];
  }
  const Node& live_c(int n) const {
    if (n < 0 || n >= (int)nodes_.size() || !nodes_[n].used || nodes_[n].root) throw PrefixError("stale prefix node");
    return nodes_[n];
  }

  PageAllocator& alloc_;
  const int P_;
  const int64_t max_pages_;
  std::vector<Node> nodes_;
  std::vector<uint32_t> epoch_;
  std::vector<int32_t> keys_;
  std::vector<int> free_;
  std::unordered_map<uint64_t, int> children_;
  std::priority_queue<HeapEntry, std::vector<HeapEntry>, std::greater<HeapEntry>> heap_;
  int64_t clock_ = 0, order_ = 0, count_ = 0;
  int64_t hits_ = 0, lookups_ = 0, hit_tokens_ = 0, evicted_ = 0;
  int roots_ = 0;
};

}  // namespace lf_host
