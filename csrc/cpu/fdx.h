// FD exchange over abstract Unix-domain sockets (see fdx.cpp).
#pragma once
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace mbx {
int fdx_listen(const std::string& name);
void fdx_send(const std::string& name, int64_t tag, const std::vector<int>& fds, int timeout_ms);
std::vector<std::pair<int64_t, std::vector<int>>> fdx_recv(int listen_fd, int count, int timeout_ms);
void fdx_close(int fd);
}  // namespace mbx
