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

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <random>
#include <string>
#include <vector>

#include "approved_fs.hpp"
#include "bpe.hpp"
#include "channel.hpp"
#include "page_allocator.hpp"

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

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: host_selftest SCRATCH_DIR\n");
    return 2;
  }
  test_allocator();
  test_bpe();
  test_channel();
  test_approved_fs(argv[1]);
  std::printf("host selftest ok\n");
  return 0;
}
