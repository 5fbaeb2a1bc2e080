// Framed control channel over a stream socket (the supervisor <-> rank link).
//
// Behaviour of the reference's process channel (internal/process: spawn +
// socketpair + exact framed I/O with deadlines, process/README.mbt.md:1-20):
// every message is one frame, written and read exactly; a peer that stops
// mid-frame or sends a corrupt header poisons the channel, and a deadline
// bounds every wait.  Frame layout (little endian):
//
//   u32 magic 'LFC1' | u32 payload length | u64 FNV-1a-64 of the payload | payload
//
// No user-space read buffering: a readable descriptor means a frame has begun,
// so callers may multiplex channels with select/poll on fileno().
#pragma once
#include <errno.h>
#include <fcntl.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <chrono>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>

namespace lf_host {

class ChannelClosed : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};
class ChannelTimeout : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

constexpr uint32_t kFrameMagic = 0x3143464Cu;  // "LFC1"

inline uint64_t fnv1a64(const uint8_t* p, size_t n) {
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

class Channel {
 public:
  // Takes its own duplicate of `fd` (close the caller's copy independently).
  Channel(int fd, uint32_t max_frame, double frame_timeout_s)
      : max_frame_(max_frame), frame_timeout_s_(frame_timeout_s) {
    fd_ = ::fcntl(fd, F_DUPFD_CLOEXEC, 0);
    if (fd_ < 0) throw ChannelClosed("cannot duplicate the channel descriptor");
  }
  ~Channel() { close(); }
  Channel(const Channel&) = delete;
  Channel& operator=(const Channel&) = delete;

  int fileno() const { return fd_; }
  bool closed() const { return fd_ < 0 || poisoned_; }

  void close() {
    if (fd_ >= 0) {
      ::close(fd_);
      fd_ = -1;
    }
  }

  // Writes one frame; the whole frame must leave within timeout_s.
  void send(const std::string& payload, double timeout_s) {
    std::lock_guard<std::mutex> g(send_mu_);
    check_open();
    if (payload.size() > max_frame_) throw std::invalid_argument("frame exceeds the channel's size limit");
    uint8_t hdr[16];
    put32(hdr, kFrameMagic);
    put32(hdr + 4, (uint32_t)payload.size());
    put64(hdr + 8, fnv1a64(reinterpret_cast<const uint8_t*>(payload.data()), payload.size()));
    const auto deadline = now() + timeout_s;
    write_exact(hdr, sizeof(hdr), deadline);
    write_exact(reinterpret_cast<const uint8_t*>(payload.data()), payload.size(), deadline);
  }

  // Waits up to timeout_s for a frame to begin (nullopt if none did); once
  // it has begun the rest must arrive within the channel's frame timeout.
  std::optional<std::string> recv(double timeout_s) {
    std::lock_guard<std::mutex> g(recv_mu_);
    check_open();
    if (!wait_io(POLLIN, now() + timeout_s)) return std::nullopt;
    const double deadline = now() + frame_timeout_s_;
    uint8_t hdr[16];
    read_exact(hdr, sizeof(hdr), deadline, /*at_start=*/true);
    const uint32_t magic = get32(hdr), len = get32(hdr + 4);
    const uint64_t sum = get64(hdr + 8);
    if (magic != kFrameMagic) poison("bad frame magic");
    if (len > max_frame_) poison("frame length exceeds the limit");
    std::string out(len, '\0');
    read_exact(reinterpret_cast<uint8_t*>(out.data()), len, deadline, false);
    if (fnv1a64(reinterpret_cast<const uint8_t*>(out.data()), len) != sum) poison("frame checksum mismatch");
    return out;
  }

 private:
  static double now() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
  }
  static void put32(uint8_t* p, uint32_t v) {
    for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(v >> (8 * i));
  }
  static void put64(uint8_t* p, uint64_t v) {
    for (int i = 0; i < 8; ++i) p[i] = (uint8_t)(v >> (8 * i));
  }
  static uint32_t get32(const uint8_t* p) {
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) v |= (uint32_t)p[i] << (8 * i);
    return v;
  }
  static uint64_t get64(const uint8_t* p) {
    uint64_t v = 0;
    for (int i = 0; i < 8; ++i) v |= (uint64_t)p[i] << (8 * i);
    return v;
  }

  void check_open() const {
    if (fd_ < 0) throw ChannelClosed("channel is closed");
    if (poisoned_) throw ChannelClosed("channel is poisoned by an earlier framing error");
  }
  [[noreturn]] void poison(const char* why) {
    poisoned_ = true;
    throw ChannelClosed(why);
  }

  // Returns false when the deadline passed first (polls at least once, so a
  // zero timeout still sees a descriptor that is ready).
  bool wait_io(short events, double deadline) {
    for (;;) {
      const double left = deadline - now();
      pollfd p{fd_, events, 0};
      const int ms = left <= 0 ? 0 : left > 3600 ? 3600 * 1000 : (int)(left * 1000) + 1;
      const int r = ::poll(&p, 1, ms);
      if (r > 0) return true;  // readable, writable, hang-up or error: the I/O call reports which
      if (r < 0 && errno != EINTR) poison("poll failed");
      if (r == 0 && left <= 0) return false;
    }
  }

  void write_exact(const uint8_t* p, size_t n, double deadline) {
    while (n > 0) {
      const ssize_t w = ::send(fd_, p, n, MSG_NOSIGNAL | MSG_DONTWAIT);
      if (w > 0) {
        p += w;
        n -= (size_t)w;
        continue;
      }
      if (w < 0 && (errno == EAGAIN || errno == EWOULDBLOCK || errno == EINTR)) {
        if (!wait_io(POLLOUT, deadline)) poison_timeout("send deadline passed mid-frame");
        continue;
      }
      poison("peer closed the channel");
    }
  }

  void read_exact(uint8_t* p, size_t n, double deadline, bool at_start) {
    size_t got = 0;
    while (got < n) {
      const ssize_t r = ::recv(fd_, p + got, n - got, MSG_DONTWAIT);
      if (r > 0) {
        got += (size_t)r;
        continue;
      }
      if (r == 0) poison(at_start && got == 0 ? "peer closed the channel" : "peer closed the channel mid-frame");
      if (errno == EAGAIN || errno == EWOULDBLOCK || errno == EINTR) {
        if (!wait_io(POLLIN, deadline)) poison_timeout("frame did not complete before its deadline");
        continue;
      }
      poison("recv failed");
    }
  }

  [[noreturn]] void poison_timeout(const char* why) {
    poisoned_ = true;
    throw ChannelTimeout(why);
  }

  int fd_ = -1;
  uint32_t max_frame_;
  double frame_timeout_s_;
  bool poisoned_ = false;
  std::mutex send_mu_, recv_mu_;
};

}  // namespace lf_host
