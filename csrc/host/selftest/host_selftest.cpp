// Self-test of the native host cores, built and run under AddressSanitizer and
// UndefinedBehaviorSanitizer by tests/test_host_sanitizers.py (CPU only):
//
//   g++ -std=c++20 -O1 -g -fsanitize=address,undefined -fno-sanitize-recover=all \
//       -I csrc/host csrc/host/selftest/host_selftest.cpp -o host_selftest && ./host_selftest DIR
//
// Exercises every public operation, the error paths included; any memory or
// undefined-behaviour error aborts with a non-zero exit status.
#include <sys/socket.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <random>
#include <string>
#include <vector>

#include "approved_fs.hpp"
#include "block_table.hpp"
#include "bpe.hpp"
#include "channel.hpp"
#include "page_allocator.hpp"
#include "prefix_tree.hpp"

using namespace lf_host;

#define CHECK(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::fprintf(stderr, "check failed: %s (line %d)\n", #c, __LINE__); \
      std::exit(1);                                                \
    }                                                              \
  } while (0)

template <class E, class F>
static bool throws(F&& f) {
  try {
    f();
  } catch (const E&) {
    return true;
  }
  return false;
}

static void test_allocator() {
  std::mt19937 rng(3);
  PageAllocator a(37, 1, 9, 1000, 1000);
  std::vector<std::pair<int, int64_t>> live;
  for (int step = 0; step < 20000; ++step) {
    const int op = rng() % 10;
    if (op < 4) {
      const int n = rng() % 5;
      if (n > a.free_page_count()) {
        CHECK(throws<OutOfPages>([&] { a.allocate_run(n); }));
      } else {
        for (auto& p : a.allocate_run(n)) live.push_back(p);
      }
    } else if (op < 8 && !live.empty()) {
      const size_t i = rng() % live.size();
      a.release_active(live[i].first, live[i].second);
      CHECK(throws<PageError>([&] { a.release_active(live[i].first, live[i].second); }));
      live.erase(live.begin() + i);
    } else if (op == 8) {
      const int64_t t = a.checkpoint();
      CHECK(throws<PageError>([&] { a.checkpoint(); }));
      const int n = std::min(2, a.free_page_count());
      auto got = a.allocate_run(n);
      if (rng() % 2) {
        a.rollback_to(t);
      } else {
        a.commit_checkpoint(t);
        for (auto& p : got) live.push_back(p);
      }
    } else if (!live.empty()) {
      auto& p = live[rng() % live.size()];
      a.retain_cached(p.first, p.second);
      a.release_cached(p.first, p.second);
    }
    a.debug_check_invariants();
  }
  CHECK(throws<PageError>([&] { a.retain_active(10000, 0); }));
  CHECK(throws<PageError>([&] { PageAllocator bad(0, 1, 5, 1, 1); }));
}

static void test_bpe() {
  // ids: a=0 b=1 c=2; merges (a,b)->3, (3,c)->4, (c,c)->5
  BpeEncoder e({{0, 1, 3}, {3, 2, 4}, {2, 2, 5}});
  CHECK((e.encode({0, 1, 2}) == std::vector<int>{4}));
  CHECK((e.encode({2, 2, 2}) == std::vector<int>{5, 2}));
  CHECK((e.encode({}) == std::vector<int>{}));
  std::mt19937 rng(5);
  for (int i = 0; i < 2000; ++i) {
    std::vector<int> s(rng() % 40);
    for (auto& x : s) x = rng() % 3;
    auto out = e.encode(s);
    CHECK(out.size() <= s.size());
  }
}

static void test_channel() {
  int sv[2];
  CHECK(::socketpair(AF_UNIX, SOCK_STREAM, 0, sv) == 0);
  {
    Channel a(sv[0], 1 << 16, 0.2), b(sv[1], 1 << 16, 0.2);
    std::string big(60000, 'q');
    a.send("hello", 1.0);
    a.send(big, 1.0);
    CHECK(*b.recv(1.0) == "hello");
    CHECK(*b.recv(1.0) == big);
    CHECK(!b.recv(0.01).has_value());
    CHECK(throws<std::invalid_argument>([&] { a.send(std::string(70000, 'x'), 1.0); }));
    // a corrupt header poisons the receiver
    const uint8_t junk[16] = {1, 2, 3, 4, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    CHECK(::write(sv[0], junk, sizeof(junk)) == (ssize_t)sizeof(junk));
    CHECK(throws<ChannelClosed>([&] { b.recv(1.0); }));
    CHECK(throws<ChannelClosed>([&] { b.recv(0.0); }));
    a.close();
    CHECK(throws<ChannelClosed>([&] { a.send("x", 1.0); }));
  }
  ::close(sv[0]);
  ::close(sv[1]);
  CHECK(::socketpair(AF_UNIX, SOCK_STREAM, 0, sv) == 0);
  {
    Channel b(sv[1], 1 << 16, 0.1);
    const uint8_t partial[8] = {0x4C, 0x46, 0x43, 0x31, 9, 0, 0, 0};  // header cut short
    CHECK(::write(sv[0], partial, sizeof(partial)) == (ssize_t)sizeof(partial));
    CHECK(throws<ChannelTimeout>([&] { b.recv(1.0); }));
  }
  ::close(sv[0]);
  ::close(sv[1]);
}

static void test_approved_fs(const std::string& dir) {
  ::mkdir((dir + "/sub").c_str(), 0755);
  {
    std::ofstream f(dir + "/sub/data.bin", std::ios::binary);
    for (int i = 0; i < 100000; ++i) f.put((char)(i % 251));
  }
  ::symlink((dir + "/sub/data.bin").c_str(), (dir + "/link").c_str());
  ApprovedRoot r(dir);
  std::vector<uint8_t> buf;
  Stamp s = r.read_snapshot("sub/data.bin", 1 << 20, [&](int64_t n) {
    buf.resize((size_t)n);
    return buf.data();
  });
  CHECK(s.size == 100000 && buf.size() == 100000 && buf[99999] == (uint8_t)(99999 % 251));
  auto none = [](int64_t) -> uint8_t* { return nullptr; };
  for (const char* bad : {"link", "../x", "/etc/passwd", "sub/../sub/data.bin", "sub//data.bin", "", "sub", "nope"})
    CHECK(throws<ApprovedFsError>([&] { r.read_snapshot(bad, 1 << 20, none); }));
  CHECK(throws<ApprovedFsError>([&] { r.read_snapshot("sub/data.bin", 10, none); }));
  CHECK(throws<ApprovedFsError>([&] { ApprovedRoot rel("relative"); }));
  r.close();
  CHECK(throws<ApprovedFsError>([&] { r.stat("sub/data.bin"); }));
}

static void test_block_tables() {
  PageAllocator a(32, 1, 1 << 20, 1 << 10, 1 << 10);
  BlockTableArena t(3, 4, 16);
  auto tid = t.allocate();
  t.append_pages(tid.first, tid.second, a.allocate_run(3));
  CHECK(t.page_count(tid.first, tid.second) == 3);
  CHECK(t.matrix_data()[tid.first * 4 + 2] == t.page_at(tid.first, tid.second, 2).first);
  CHECK(t.resolve_token_position(tid.first, tid.second, 33).second == 1);
  CHECK(throws<BlockTableError>([&] { t.resolve_token_position(tid.first, tid.second, 48); }));
  CHECK(throws<BlockTableError>([&] { t.append_pages(tid.first, tid.second, a.allocate_run(2)); }));
  t.checkpoint();
  t.note(tid.first);
  auto extra = a.allocate_run(1);
  t.append_pages(tid.first, tid.second, extra);
  t.rollback();
  CHECK(t.page_count(tid.first, tid.second) == 3 && t.matrix_data()[tid.first * 4 + 3] == 0);
  a.release_active(extra[0].first, extra[0].second);
  CHECK(t.truncate(tid.first, tid.second, 1, &a).size() == 2);
  CHECK(throws<BlockTableError>([&] { t.release(tid.first, tid.second); }));
  t.reset_and_release(tid.first, tid.second, &a);
  CHECK(throws<BlockTableError>([&] { t.page_count(tid.first, tid.second); }));
  t.debug_check_invariants();
  a.debug_check_invariants();
  for (int i = 0; i < 3; ++i) t.allocate();
  CHECK(throws<BlockTableError>([&] { t.allocate(); }));
}

static void test_prefix_tree() {
  const int P = 2;
  PageAllocator a(64, 1, 1 << 20, 1 << 10, 1 << 10);
  PrefixTree tree(a, P, 40);
  const int r0 = tree.new_root(), r1 = tree.new_root();
  std::mt19937 rng(7);
  std::vector<std::vector<int>> held;
  for (int step = 0; step < 3000; ++step) {
    const int op = rng() % 5;
    const int root = (rng() & 1) ? r0 : r1;
    std::vector<int32_t> toks(rng() % 10);
    for (auto& x : toks) x = (int32_t)(rng() % 3);
    if (op <= 1) {
      const int n = std::min<int>((int)(toks.size() / P), a.free_page_count());
      auto pages = a.allocate_run(n);
      tree.insert(root, toks.data(), (int64_t)toks.size(), pages);
      for (auto& p : pages) a.release_active(p.first, p.second);
    } else if (op == 2) {
      auto nodes = tree.lookup(root, toks.data(), (int64_t)toks.size(), -1);
      CHECK(tree.pages_of(nodes).size() == nodes.size());
      if (!nodes.empty() && (rng() & 1)) {
        tree.retain(nodes);
        held.push_back(nodes);
      }
    } else if (op == 3 && !held.empty()) {
      tree.release(held.back());
      held.pop_back();
    } else {
      tree.evict(rng() % 5);
    }
    if (step % 500 == 0) tree.debug_check_invariants();
  }
  for (auto& h : held) tree.release(h);
  tree.evict(1 << 30);
  CHECK(tree.page_count() == 0 && a.free_page_count() == 64);
  CHECK(throws<PrefixError>([&] { tree.retain({12345}); }));
  CHECK(throws<PrefixError>([&] { tree.lookup(999, nullptr, 0, -1); }));
  tree.debug_check_invariants();
  a.debug_check_invariants();
}

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: host_selftest SCRATCH_DIR\n");
    return 2;
  }
  test_allocator();
  test_block_tables();
  test_prefix_tree();
  test_bpe();
  test_channel();
  test_approved_fs(argv[1]);
  std::printf("host selftest ok\n");
  return 0;
}
