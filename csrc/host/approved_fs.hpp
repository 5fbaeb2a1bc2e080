// Approved filesystem root: component-by-component, no-follow file access.
//
// Behaviour of the reference's internal/approved_fs (traversal.c: openat with
// O_NOFOLLOW and a type check per component; identity and snapshot stamps)
// and runtime/approved_fs/api.mbt:67-81.  A deployment names an absolute
// root; a relative locator is resolved one component at a time with
// openat(dir_fd, name, O_NOFOLLOW), so no symlink, "..", "." or absolute
// component can leave the root.  A snapshot read returns the file's bytes
// with a (device, inode, size, mtime, ctime) stamp and fails if the stamp
// changed while the file was read.  Reads go straight into the caller's
// buffer (for weights: a pinned staging buffer), with the GIL released by the
// binding.
#pragma once
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

namespace lf_host {

class ApprovedFsError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

struct Stamp {
  uint64_t dev, ino;
  int64_t size, mtime_ns, ctime_ns;
  bool operator==(const Stamp& o) const {
    return dev == o.dev && ino == o.ino && size == o.size && mtime_ns == o.mtime_ns && ctime_ns == o.ctime_ns;
  }
};

inline Stamp stamp_of(const struct stat& st) {
  return Stamp{(uint64_t)st.st_dev, (uint64_t)st.st_ino, (int64_t)st.st_size,
               (int64_t)st.st_mtim.tv_sec * 1000000000ll + st.st_mtim.tv_nsec,
               (int64_t)st.st_ctim.tv_sec * 1000000000ll + st.st_ctim.tv_nsec};
}

class FdGuard {
 public:
  explicit FdGuard(int fd = -1) : fd_(fd) {}
  ~FdGuard() {
    if (fd_ >= 0) ::close(fd_);
  }
  FdGuard(const FdGuard&) = delete;
  FdGuard& operator=(const FdGuard&) = delete;
  int get() const { return fd_; }

 private:
  int fd_;
};

class ApprovedRoot {
 public:
  explicit ApprovedRoot(const std::string& path) {
    if (path.empty() || path[0] != '/') throw ApprovedFsError("approved root must be an absolute path");
    fd_ = ::open(path.c_str(), O_RDONLY | O_DIRECTORY | O_NOFOLLOW | O_CLOEXEC);
    if (fd_ < 0) throw ApprovedFsError(std::string("cannot open approved root: ") + std::strerror(errno));
    struct stat st;
    ::fstat(fd_, &st);
    identity_ = stamp_of(st);
  }
  ~ApprovedRoot() { close(); }
  ApprovedRoot(const ApprovedRoot&) = delete;
  ApprovedRoot& operator=(const ApprovedRoot&) = delete;

  void close() {
    if (fd_ >= 0) {
      ::close(fd_);
      fd_ = -1;
    }
  }
  const Stamp& identity() const { return identity_; }

  // Opens a locator as a regular file (caller owns the descriptor).
  int open_file(const std::string& locator) const {
    if (fd_ < 0) throw ApprovedFsError("approved root is closed");
    std::vector<std::string> parts;
    if (locator.empty() || locator[0] == '/') throw bad_locator();
    size_t s = 0;
    for (;;) {
      const size_t e = locator.find('/', s);
      parts.push_back(locator.substr(s, e == std::string::npos ? std::string::npos : e - s));
      if (e == std::string::npos) break;
      s = e + 1;
    }
    for (const auto& p : parts)
      if (p.empty() || p == "." || p == "..") throw bad_locator();
    int dfd = fd_;
    std::vector<int> opened;
    auto cleanup = [&] {
      for (int f : opened) ::close(f);
    };
    for (size_t i = 0; i + 1 < parts.size(); ++i) {
      const int nfd = ::openat(dfd, parts[i].c_str(), O_RDONLY | O_DIRECTORY | O_NOFOLLOW | O_CLOEXEC);
      if (nfd < 0) {
        const int err = errno;
        cleanup();
        throw ApprovedFsError(std::string("cannot open locator: ") + std::strerror(err));
      }
      opened.push_back(nfd);
      dfd = nfd;
    }
    // O_NONBLOCK: opening a FIFO must not wait for a writer (it is rejected below)
    const int fd = ::openat(dfd, parts.back().c_str(), O_RDONLY | O_NOFOLLOW | O_CLOEXEC | O_NONBLOCK);
    const int err = errno;
    cleanup();
    if (fd < 0) throw ApprovedFsError(std::string("cannot open locator: ") + std::strerror(err));
    struct stat st;
    if (::fstat(fd, &st) != 0 || !S_ISREG(st.st_mode)) {
      ::close(fd);
      throw ApprovedFsError("locator is not a regular file");
    }
    ::fcntl(fd, F_SETFL, ::fcntl(fd, F_GETFL) & ~O_NONBLOCK);
    return fd;
  }

  // Stats a locator (the size decides the caller's buffer).
  Stamp stat(const std::string& locator) const {
    FdGuard fd(open_file(locator));
    struct stat st;
    ::fstat(fd.get(), &st);
    return stamp_of(st);
  }

  // Reads the whole file.  `alloc` is called
  // with the size once it is known and returns the destination.
  Stamp read_snapshot(const std::string& locator, int64_t max_bytes,
                      const std::function<uint8_t*(int64_t)>& alloc) const {
    FdGuard fd(open_file(locator));
    struct stat st;
    ::fstat(fd.get(), &st);
    const Stamp before = stamp_of(st);
    if (before.size > max_bytes) throw ApprovedFsError("file exceeds the size limit");
    uint8_t* dst = alloc(before.size);
    int64_t off = 0;
    while (off < before.size) {
      const size_t want = (size_t)std::min<int64_t>(1ll << 26, before.size - off);
      const ssize_t r = ::pread(fd.get(), dst + off, want, off);
      if (r < 0) {
        if (errno == EINTR) continue;
        throw ApprovedFsError(std::string("read failed: ") + std::strerror(errno));
      }
      if (r == 0) break;
      off += r;
    }
    ::fstat(fd.get(), &st);
    if (!(stamp_of(st) == before) || off != before.size) throw ApprovedFsError("file changed while it was read");
    return before;
  }

 private:
  static ApprovedFsError bad_locator() {
    return ApprovedFsError("locator must be a relative path without '.', '..' or empty components");
  }
  int fd_ = -1;
  Stamp identity_{};
};

}  // namespace lf_host
