// ZMTP 3.0 SUB client (see zmtp.h).
#include "zmtp.h"

#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>

#include "net.h"

namespace ib {

ZmtpSub::~ZmtpSub() { close(); }

void ZmtpSub::close() {
  if (fd_ >= 0) {
    ::close(fd_);
    fd_ = -1;
  }
}

bool ZmtpSub::read_n(char* dst, size_t n, int timeout_ms) {
  while (n > 0) {
    if (timeout_ms >= 0) {
      pollfd pf{fd_, POLLIN, 0};
      int r = ::poll(&pf, 1, timeout_ms);
      if (r == 0) return false;
      if (r < 0 && errno != EINTR) return false;
      if (r < 0) continue;
    }
    ssize_t r = ::recv(fd_, dst, n, 0);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    dst += r;
    n -= static_cast<size_t>(r);
  }
  return true;
}

bool ZmtpSub::send_frame(const std::string& body, bool command, bool more) {
  std::string f;
  unsigned char flags = (more ? 0x01 : 0) | (command ? 0x04 : 0);
  if (body.size() > 255) {
    flags |= 0x02;
    f.push_back(static_cast<char>(flags));
    for (int k = 7; k >= 0; --k) f.push_back(static_cast<char>((body.size() >> (8 * k)) & 0xFF));
  } else {
    f.push_back(static_cast<char>(flags));
    f.push_back(static_cast<char>(body.size()));
  }
  f += body;
  return write_all(fd_, f);
}

int ZmtpSub::read_frame(std::string* body, bool* command, bool* more, int timeout_ms) {
  unsigned char flags;
  if (timeout_ms >= 0) {
    pollfd pf{fd_, POLLIN, 0};
    int r = ::poll(&pf, 1, timeout_ms);
    if (r == 0) return 0;
    if (r < 0) return errno == EINTR ? 0 : -1;
  }
  if (!read_n(reinterpret_cast<char*>(&flags), 1, 30000)) return -1;
  uint64_t size = 0;
  if (flags & 0x02) {
    unsigned char b[8];
    if (!read_n(reinterpret_cast<char*>(b), 8, 30000)) return -1;
    for (int k = 0; k < 8; ++k) size = (size << 8) | b[k];
  } else {
    unsigned char b;
    if (!read_n(reinterpret_cast<char*>(&b), 1, 30000)) return -1;
    size = b;
  }
  if (size > (1ull << 31)) return -1;
  body->resize(size);
  if (size && !read_n(&(*body)[0], size, 30000)) return -1;
  *command = flags & 0x04;
  *more = flags & 0x01;
  return 1;
}

bool ZmtpSub::connect(const std::string& endpoint, const std::string& topic, int timeout_ms) {
  close();
  Url u;
  if (endpoint.compare(0, 6, "tcp://") != 0 || !parse_url(endpoint, &u)) {
    err_ = "only tcp:// endpoints are supported";
    return false;
  }
  fd_ = tcp_connect(u.host, u.port, timeout_ms);
  if (fd_ < 0) {
    err_ = "connect failed";
    return false;
  }
  // greeting: signature (10), version 3.0 (2), mechanism "NULL" (20), as-server 0, filler (31)
  char g[64];
  std::memset(g, 0, sizeof(g));
  g[0] = static_cast<char>(0xFF);
  g[9] = 0x7F;
  g[10] = 3;
  g[11] = 0;
  std::memcpy(g + 12, "NULL", 4);
  if (!write_all(fd_, g, sizeof(g))) { err_ = "greeting send failed"; close(); return false; }
  char pg[64];
  if (!read_n(pg, 64, timeout_ms) || static_cast<unsigned char>(pg[0]) != 0xFF || pg[9] != 0x7F || pg[10] < 3) {
    err_ = "bad peer greeting";
    close();
    return false;
  }
  // READY command with Socket-Type = SUB
  std::string ready;
  ready.push_back(5);
  ready += "READY";
  const std::string name = "Socket-Type", value = "SUB";
  ready.push_back(static_cast<char>(name.size()));
  ready += name;
  for (int k = 3; k >= 0; --k) ready.push_back(static_cast<char>((value.size() >> (8 * k)) & 0xFF));
  ready += value;
  if (!send_frame(ready, true, false)) { err_ = "READY send failed"; close(); return false; }
  // the peer's READY
  while (true) {
    std::string body;
    bool cmd, more;
    int r = read_frame(&body, &cmd, &more, timeout_ms);
    if (r <= 0) { err_ = "no READY from peer"; close(); return false; }
    if (cmd && body.size() >= 6 && body[0] == 5 && body.compare(1, 5, "READY") == 0) break;
    if (cmd && body.size() >= 6 && body[0] == 5 && body.compare(1, 5, "ERROR") == 0) {
      err_ = "peer ERROR";
      close();
      return false;
    }
  }
  // subscription: a message whose first byte is 1, then the topic prefix
  std::string sub(1, '\x01');
  sub += topic;
  if (!send_frame(sub, false, false)) { err_ = "subscribe failed"; close(); return false; }
  return true;
}

int ZmtpSub::recv(std::vector<std::string>* frames, int timeout_ms) {
  if (fd_ < 0) return -1;
  frames->clear();
  while (true) {
    std::string body;
    bool cmd = false, more = false;
    int r = read_frame(&body, &cmd, &more, frames->empty() ? timeout_ms : 30000);
    if (r == 0) return frames->empty() ? 0 : -1;
    if (r < 0) {
      close();
      return -1;
    }
    if (cmd) continue;
    frames->push_back(std::move(body));
    if (!more) return 1;
  }
}

}  // namespace ib
