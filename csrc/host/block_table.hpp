// Per-request block tables: logical page -> physical PageId, in an arena of
// generational table slots (reference semantics of kv/block_table/arena.mbt:
// 12-369 and allocation_checkpoint.mbt:17-166).
//
// Besides the (index, generation) page ids, the arena owns a dense row-major
// int32 [capacity][max_pages] matrix of physical page indices (generations
// stripped, as they are before a step is uploaded); Python sees it as a numpy
// view and slices it straight into the packed step block.  A checkpoint
// remembers each noted table's length; rollback cuts the suffixes appended
// since then (the page allocator's own rollback reclaims those pages).
//
// Exact restatement of the Python reference class BlockTableArena
// (lunaflux_b200/kv/block_table.py), which the tests run against it.
#pragma once
#include <cstdint>
#include <map>
#include <stdexcept>
#include <utility>
#include <vector>

#include "page_allocator.hpp"

namespace lf_host {

class BlockTableError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

class BlockTableArena {
 public:
  using Page = std::pair<int, int64_t>;

  BlockTableArena(int capacity, int max_pages, int tokens_per_page)
      : cap_(capacity), maxp_(max_pages), P_(tokens_per_page) {
    if (capacity <= 0 || max_pages <= 0 || tokens_per_page <= 0) throw BlockTableError("arena dimensions must be positive");
    gen_.assign(cap_, 0);
    live_.assign(cap_, 0);
    pages_.resize(cap_);
    matrix_.assign((size_t)cap_ * maxp_, 0);
    for (int s = cap_ - 1; s >= 0; --s) free_.push_back(s);
  }

  int capacity() const { return cap_; }
  int max_pages() const { return maxp_; }
  int tokens_per_page() const { return P_; }
  int free_table_count() const { return (int)free_.size(); }
  int allocated_table_count() const { return cap_ - (int)free_.size(); }
  int32_t* matrix_data() { return matrix_.data(); }

  std::pair<int, int64_t> allocate() {
    if (free_.empty()) throw BlockTableError("no free block table");
    const int s = free_.back();
    free_.pop_back();
    live_[s] = 1;
    pages_[s].clear();
    return {s, gen_[s]};
  }

  void release(int idx, int64_t g) {
    const int s = slot(idx, g);
    if (!pages_[s].empty()) throw BlockTableError("table still owns pages; use reset_and_release");
    live_[s] = 0;
    ++gen_[s];
    free_.push_back(s);
  }

  int page_count(int idx, int64_t g) const { return (int)pages_[slot(idx, g)].size(); }
  std::vector<Page> pages(int idx, int64_t g) const { return pages_[slot(idx, g)]; }

  void append_pages(int idx, int64_t g, const std::vector<Page>& pids) {
    const int s = slot(idx, g);
    auto& v = pages_[s];
    const size_t n = v.size();
    if (n + pids.size() > (size_t)maxp_) throw BlockTableError("block table full");
    int32_t* row = matrix_.data() + (size_t)s * maxp_;
    for (size_t i = 0; i < pids.size(); ++i) {
      v.push_back(pids[i]);
      row[n + i] = pids[i].first;
    }
  }

  Page page_at(int idx, int64_t g, int logical) const {
    const auto& v = pages_[slot(idx, g)];
    if (logical < 0 || logical >= (int)v.size()) throw BlockTableError("logical page out of range");
    return v[logical];
  }

  // (physical page index, offset in the page) of a token position
  std::pair<int, int> resolve_token_position(int idx, int64_t g, int64_t position) const {
    const auto& v = pages_[slot(idx, g)];
    if (position < 0) throw BlockTableError("negative position");
    const int64_t lp = position / P_;
    if (lp >= (int64_t)v.size()) throw BlockTableError("position beyond the table");
    return {v[lp].first, (int)(position % P_)};
  }

  // Drops the pages from `keep` on (releasing their active reference when an
  // allocator is given) and returns them.
  std::vector<Page> truncate(int idx, int64_t g, int keep, PageAllocator* alloc) {
    const int s = slot(idx, g);
    auto& v = pages_[s];
    if (keep < 0) throw BlockTableError("negative length");
    if (keep >= (int)v.size()) return {};
    std::vector<Page> dropped(v.begin() + keep, v.end());
    // preflight: a release that would fail throws here, with the table and
    // the allocator untouched
    if (alloc != nullptr) alloc->check_release_active(dropped);
    v.resize(keep);
    int32_t* row = matrix_.data() + (size_t)s * maxp_;
    for (size_t i = 0; i < dropped.size(); ++i) row[keep + i] = 0;
    if (alloc != nullptr)
      for (const auto& p : dropped) alloc->release_active(p.first, p.second);
    return dropped;
  }

  void reset_and_release(int idx, int64_t g, PageAllocator* alloc) {
    truncate(idx, g, 0, alloc);
    release(idx, g);
  }

  void checkpoint() {
    if (ckpt_open_) throw BlockTableError("checkpoint already open");
    ckpt_open_ = true;
    ckpt_.clear();
  }
  void note(int idx) {
    if (ckpt_open_ && idx >= 0 && idx < cap_ && ckpt_.find(idx) == ckpt_.end()) ckpt_[idx] = pages_[idx].size();
  }
  void commit_checkpoint() {
    ckpt_open_ = false;
    ckpt_.clear();
  }
  void rollback() {
    for (const auto& [s, n] : ckpt_) {
      auto& v = pages_[s];
      if (v.size() > n) {
        int32_t* row = matrix_.data() + (size_t)s * maxp_;
        for (size_t i = n; i < v.size(); ++i) row[i] = 0;
        v.resize(n);
      }
    }
    ckpt_open_ = false;
    ckpt_.clear();
  }

  void debug_check_invariants() const {
    std::vector<uint8_t> in_free(cap_, 0);
    for (int s : free_) {
      if (s < 0 || s >= cap_ || in_free[s] || live_[s]) throw BlockTableError("free table list");
      in_free[s] = 1;
    }
    for (int s = 0; s < cap_; ++s) {
      if (!live_[s] && !in_free[s]) throw BlockTableError("table neither live nor free");
      if (!live_[s] && !pages_[s].empty()) throw BlockTableError("free table owns pages");
      const int32_t* row = matrix_.data() + (size_t)s * maxp_;
      for (int i = 0; i < maxp_; ++i) {
        const int32_t want = i < (int)pages_[s].size() ? pages_[s][i].first : 0;
        if (row[i] != want) throw BlockTableError("matrix does not mirror the page ids");
      }
    }
  }

 private:
  int slot(int idx, int64_t g) const {
    if (idx < 0 || idx >= cap_ || !live_[idx] || gen_[idx] != g) throw BlockTableError("stale or unknown table id");
    return idx;
  }

  int cap_, maxp_, P_;
  std::vector<int64_t> gen_;
  std::vector<uint8_t> live_;
  std::vector<std::vector<Page>> pages_;
  std::vector<int32_t> matrix_;
  std::vector<int> free_;
  bool ckpt_open_ = false;
  std::map<int, size_t> ckpt_;
};

}  // namespace lf_host
