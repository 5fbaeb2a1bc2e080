// Generational KV page allocator (reference semantics of
// kv/page_allocator/allocator.mbt:13-302 and allocation_checkpoint.mbt:7-107):
// (index, generation) ids, separate active and cached reference counts, an
// FIFO free queue, retirement at the terminal generation, one exclusive
// checkpoint with exact rollback.  O(1) per page.  Exact restatement of the
// Python reference class PyPageAllocator (lunaflux_b200/kv/page_allocator.py).
#pragma once
#include <algorithm>
#include <cstdint>
#include <deque>
#include <stdexcept>
#include <utility>
#include <vector>

namespace lf_host {


class PageError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};
class OutOfPages : public PageError {
 public:
  using PageError::PageError;
};

class PageAllocator {
 public:
  enum State : uint8_t { kFree = 0, kAllocated = 1, kRetired = 2 };

  PageAllocator(int capacity, int first_index, int64_t max_generation, int max_active, int max_cached)
      : cap_(capacity), first_(first_index), max_gen_(max_generation), max_active_(max_active), max_cached_(max_cached) {
    if (capacity <= 0) throw PageError("capacity must be positive");
    gen_.assign(cap_, 0);
    state_.assign(cap_, kFree);
    active_.assign(cap_, 0);
    cached_.assign(cap_, 0);
    for (int i = 0; i < cap_; ++i) free_.push_back(i);
  }

  int free_page_count() const { return (int)free_.size(); }
  int allocated_page_count() const { return allocated_; }
  int retired_page_count() const { return retired_; }
  int capacity() const { return cap_; }

  std::vector<std::pair<int, int64_t>> allocate_run(int n) {
    if (n < 0) throw PageError("negative run");
    if (n > (int)free_.size()) throw OutOfPages("not enough free pages");
    std::vector<std::pair<int, int64_t>> out;
    out.reserve(n);
    for (int i = 0; i < n; ++i) {
      const int s = free_.front();
      free_.pop_front();
      if (ckpt_open_) {
        popped_.push_back(s);
        prev_gen_.push_back(gen_[s]);
      }
      state_[s] = kAllocated;
      active_[s] = 1;
      ++allocated_;
      out.emplace_back(s + first_, gen_[s]);
    }
    return out;
  }

  void retain_active(int idx, int64_t g) {
    no_ckpt();
    const int s = slot(idx, g);
    if (active_[s] >= max_active_) throw PageError("active reference limit");
    ++active_[s];
  }
  void release_active(int idx, int64_t g) {
    no_ckpt();
    const int s = slot(idx, g);
    if (active_[s] <= 0) throw PageError("no active reference to release");
    --active_[s];
    maybe_free(s);
  }
  void retain_cached(int idx, int64_t g) {
    no_ckpt();
    const int s = slot(idx, g);
    if (cached_[s] >= max_cached_) throw PageError("cached reference limit");
    ++cached_[s];
  }
  void release_cached(int idx, int64_t g) {
    no_ckpt();
    const int s = slot(idx, g);
    if (cached_[s] <= 0) throw PageError("no cached reference to release");
    --cached_[s];
    maybe_free(s);
  }
  // Throws, changing nothing, unless release_active could run once for every
  // entry of `pages` (a page listed n times needs n active references).
  void check_release_active(const std::vector<std::pair<int, int64_t>>& pages) const {
    no_ckpt();
    std::vector<std::pair<int, int>> need;  // (slot, count), sorted below
    need.reserve(pages.size());
    for (const auto& p : pages) need.emplace_back(slot(p.first, p.second), 1);
    std::sort(need.begin(), need.end());
    for (size_t i = 0; i < need.size();) {
      size_t j = i;
      while (j < need.size() && need[j].first == need[i].first) ++j;
      if (active_[need[i].first] < (int)(j - i)) throw PageError("no active reference to release");
      i = j;
    }
  }
  int active_reference_count(int idx, int64_t g) const { return active_[slot(idx, g)]; }
  int cached_reference_count(int idx, int64_t g) const { return cached_[slot(idx, g)]; }
  bool validate_active(int idx, int64_t g) const {
    const int s = idx - first_;
    return s >= 0 && s < cap_ && gen_[s] == g && state_[s] == kAllocated && active_[s] > 0;
  }

  int64_t checkpoint() {
    if (ckpt_open_) throw PageError("a checkpoint is already open");
    ckpt_open_ = true;
    popped_.clear();
    prev_gen_.clear();
    return ++ckpt_seq_;
  }
  void commit_checkpoint(int64_t token) {
    if (!ckpt_open_ || token != ckpt_seq_) throw PageError("checkpoint token mismatch");
    ckpt_open_ = false;
  }
  void rollback_to(int64_t token) {
    if (!ckpt_open_ || token != ckpt_seq_) throw PageError("checkpoint token mismatch");
    for (size_t i = popped_.size(); i-- > 0;) {
      const int s = popped_[i];
      state_[s] = kFree;
      active_[s] = 0;
      gen_[s] = prev_gen_[i];
      --allocated_;
      free_.push_front(s);
    }
    ckpt_open_ = false;
  }

  std::vector<int> free_queue() const { return std::vector<int>(free_.begin(), free_.end()); }

  void debug_check_invariants() const {
    std::vector<uint8_t> in_free(cap_, 0);
    for (int s : free_) {
      if (in_free[s]) throw PageError("duplicate in free queue");
      in_free[s] = 1;
    }
    int n_alloc = 0, n_ret = 0;
    for (int s = 0; s < cap_; ++s) {
      if (state_[s] == kFree) {
        if (!in_free[s] || active_[s] || cached_[s]) throw PageError("free page invariant");
      } else if (state_[s] == kAllocated) {
        if (in_free[s] || (active_[s] <= 0 && cached_[s] <= 0)) throw PageError("allocated page invariant");
        ++n_alloc;
      } else {
        if (in_free[s]) throw PageError("retired page in free queue");
        ++n_ret;
      }
    }
    if (n_alloc != allocated_ || n_ret != retired_ || (int)free_.size() + n_alloc + n_ret != cap_)
      throw PageError("page counters");
  }

 private:
  int slot(int idx, int64_t g) const {
    const int s = idx - first_;
    if (s < 0 || s >= cap_ || gen_[s] != g || state_[s] != kAllocated) throw PageError("stale or unknown page id");
    return s;
  }
  void no_ckpt() const {
    if (ckpt_open_) throw PageError("reference counts are frozen while a checkpoint is open");
  }
  void maybe_free(int s) {
    if (active_[s] == 0 && cached_[s] == 0) {
      --allocated_;
      if (gen_[s] >= max_gen_) {
        state_[s] = kRetired;
        ++retired_;
      } else {
        ++gen_[s];
        state_[s] = kFree;
        free_.push_back(s);
      }
    }
  }

  int cap_, first_;
  int64_t max_gen_;
  int max_active_, max_cached_;
  std::vector<int64_t> gen_;
  std::vector<uint8_t> state_;
  std::vector<int> active_, cached_;
  std::deque<int> free_;
  int allocated_ = 0, retired_ = 0;
  bool ckpt_open_ = false;
  int64_t ckpt_seq_ = 0;
  std::vector<int> popped_;
  std::vector<int64_t> prev_gen_;
};

}  // namespace lf_host
