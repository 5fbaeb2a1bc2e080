// Byte-level BPE merge loop of tokenizer/encode.mbt on token ids: pick the
// best-ranked adjacent pair over the whole sequence, merge every
// non-overlapping occurrence left to right, repeat.  Exact restatement of
// Tokenizer._bpe_reference (lunaflux_b200/tokenizer/bpe.py).
#pragma once
#include <cstdint>
#include <tuple>
#include <unordered_map>
#include <utility>
#include <vector>

namespace lf_host {

class BpeEncoder {
 public:
  // merges: (left id, right id, merged id) in rank order
  explicit BpeEncoder(const std::vector<std::tuple<int, int, int>>& merges) {
    for (size_t r = 0; r < merges.size(); ++r) {
      const auto& m = merges[r];
      table_.emplace(key(std::get<0>(m), std::get<1>(m)), std::make_pair((int)r, std::get<2>(m)));
    }
  }

  std::vector<int> encode(std::vector<int> syms) const {
    while (syms.size() > 1) {
      int best_rank = -1, best_id = -1, a = -1, b = -1;
      for (size_t i = 0; i + 1 < syms.size(); ++i) {
        auto it = table_.find(key(syms[i], syms[i + 1]));
        if (it != table_.end() && (best_rank < 0 || it->second.first < best_rank)) {
          best_rank = it->second.first;
          best_id = it->second.second;
          a = syms[i];
          b = syms[i + 1];
        }
      }
      if (best_rank < 0) break;
      std::vector<int> out;
      out.reserve(syms.size());
      for (size_t i = 0; i < syms.size();) {
        if (i + 1 < syms.size() && syms[i] == a && syms[i + 1] == b) {
          out.push_back(best_id);
          i += 2;
        } else {
          out.push_back(syms[i]);
          i += 1;
        }
      }
      syms.swap(out);
    }
    return syms;
  }

 private:
  static uint64_t key(int a, int b) { return ((uint64_t)(uint32_t)a << 32) | (uint32_t)b; }
  std::unordered_map<uint64_t, std::pair<int, int>> table_;
};

}  // namespace lf_host
