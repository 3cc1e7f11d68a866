// File-descriptor exchange between the ranks of one node.
//
// cuMem POSIX-FD handles (and NVLS multicast handles) are plain file
// descriptors; they only mean something in another process once passed over a
// Unix-domain socket with SCM_RIGHTS. Each rank listens on an abstract-
// namespace socket (no filesystem entry, gone when the process exits); peers
// connect and send (tag, fds...) in one message. The reference exchanges
// 64-byte cudaIpc handles through torch.distributed.all_gather_object
// (sglang/mailbox_all_reduce.py:116); FDs cannot travel that way.
#include <errno.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <time.h>
#include <unistd.h>

#include <chrono>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "fdx.h"

namespace mbx {
namespace {

constexpr int kMaxFds = 16;

sockaddr_un make_addr(const std::string& name, socklen_t* len) {
  if (name.size() + 1 > sizeof(sockaddr_un::sun_path)) throw std::runtime_error("fdx: socket name too long");
  sockaddr_un a;
  std::memset(&a, 0, sizeof(a));
  a.sun_family = AF_UNIX;
  a.sun_path[0] = '\0';  // abstract namespace
  std::memcpy(a.sun_path + 1, name.data(), name.size());
  *len = (socklen_t)(offsetof(sockaddr_un, sun_path) + 1 + name.size());
  return a;
}

std::string errno_str(const char* what) { return std::string("fdx: ") + what + ": " + std::strerror(errno); }

}  // namespace

int fdx_listen(const std::string& name) {
  int s = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (s < 0) throw std::runtime_error(errno_str("socket"));
  socklen_t len;
  sockaddr_un a = make_addr(name, &len);
  if (::bind(s, (sockaddr*)&a, len) != 0) {
    int e = errno;
    ::close(s);
    errno = e;
    throw std::runtime_error(errno_str("bind"));
  }
  if (::listen(s, 64) != 0) {
    int e = errno;
    ::close(s);
    errno = e;
    throw std::runtime_error(errno_str("listen"));
  }
  return s;
}

void fdx_send(const std::string& name, int64_t tag, const std::vector<int>& fds, int timeout_ms) {
  if (fds.size() > (size_t)kMaxFds) throw std::runtime_error("fdx: too many fds");
  socklen_t len;
  sockaddr_un a = make_addr(name, &len);
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  int s = -1;
  while (true) {
    s = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (s < 0) throw std::runtime_error(errno_str("socket"));
    if (::connect(s, (sockaddr*)&a, len) == 0) break;
    ::close(s);
    s = -1;
    if (std::chrono::steady_clock::now() > deadline) throw std::runtime_error("fdx: connect to '" + name + "' timed out");
    std::this_thread::sleep_for(std::chrono::milliseconds(5));
  }
  struct {
    int64_t tag;
    int32_t nfds;
  } payload{tag, (int32_t)fds.size()};
  iovec iov{&payload, sizeof(payload)};
  alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int) * kMaxFds)];
  std::memset(ctrl, 0, sizeof(ctrl));
  msghdr msg;
  std::memset(&msg, 0, sizeof(msg));
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  if (!fds.empty()) {
    msg.msg_control = ctrl;
    msg.msg_controllen = CMSG_SPACE(sizeof(int) * fds.size());
    cmsghdr* cm = CMSG_FIRSTHDR(&msg);
    cm->cmsg_level = SOL_SOCKET;
    cm->cmsg_type = SCM_RIGHTS;
    cm->cmsg_len = CMSG_LEN(sizeof(int) * fds.size());
    std::memcpy(CMSG_DATA(cm), fds.data(), sizeof(int) * fds.size());
  }
  ssize_t n = ::sendmsg(s, &msg, MSG_NOSIGNAL);
  int e = errno;
  ::close(s);
  errno = e;
  if (n != (ssize_t)sizeof(payload)) throw std::runtime_error(errno_str("sendmsg"));
}

std::vector<std::pair<int64_t, std::vector<int>>> fdx_recv(int listen_fd, int count, int timeout_ms) {
  std::vector<std::pair<int64_t, std::vector<int>>> out;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  while ((int)out.size() < count) {
    const int left =
        (int)std::chrono::duration_cast<std::chrono::milliseconds>(deadline - std::chrono::steady_clock::now()).count();
    if (left <= 0) throw std::runtime_error("fdx: receive timed out (" + std::to_string(out.size()) + "/" +
                                            std::to_string(count) + " peers)");
    pollfd p{listen_fd, POLLIN, 0};
    int pr = ::poll(&p, 1, left);
    if (pr < 0) {
      if (errno == EINTR) continue;
      throw std::runtime_error(errno_str("poll"));
    }
    if (pr == 0) continue;
    int c = ::accept4(listen_fd, nullptr, nullptr, SOCK_CLOEXEC);
    if (c < 0) {
      if (errno == EINTR || errno == EAGAIN) continue;
      throw std::runtime_error(errno_str("accept"));
    }
    struct {
      int64_t tag;
      int32_t nfds;
    } payload{};
    iovec iov{&payload, sizeof(payload)};
    alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int) * kMaxFds)];
    msghdr msg;
    std::memset(&msg, 0, sizeof(msg));
    msg.msg_iov = &iov;
    msg.msg_iovlen = 1;
    msg.msg_control = ctrl;
    msg.msg_controllen = sizeof(ctrl);
    ssize_t n = ::recvmsg(c, &msg, MSG_CMSG_CLOEXEC);
    ::close(c);
    if (n != (ssize_t)sizeof(payload)) throw std::runtime_error(errno_str("recvmsg"));
    std::vector<int> fds;
    for (cmsghdr* cm = CMSG_FIRSTHDR(&msg); cm; cm = CMSG_NXTHDR(&msg, cm)) {
      if (cm->cmsg_level == SOL_SOCKET && cm->cmsg_type == SCM_RIGHTS) {
        const int k = (int)((cm->cmsg_len - CMSG_LEN(0)) / sizeof(int));
        for (int i = 0; i < k; ++i) {
          int fd;
          std::memcpy(&fd, CMSG_DATA(cm) + i * sizeof(int), sizeof(int));
          fds.push_back(fd);
        }
      }
    }
    if ((int)fds.size() != payload.nfds) throw std::runtime_error("fdx: fd count mismatch");
    out.emplace_back(payload.tag, std::move(fds));
  }
  return out;
}

void fdx_close(int fd) {
  if (fd >= 0) ::close(fd);
}

}  // namespace mbx
