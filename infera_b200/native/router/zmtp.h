// ZMTP 3.0 SUB client over TCP (rfc.zeromq.org/spec/23 and /37), enough to
// follow a PUB socket: greeting with the NULL mechanism, READY with
// Socket-Type SUB, a subscription message, then multipart messages.
// Commands the peer sends after the handshake (PING etc.) are skipped.
#pragma once

#include <string>
#include <vector>

namespace ib {

class ZmtpSub {
 public:
  ZmtpSub() = default;
  ~ZmtpSub();
  ZmtpSub(const ZmtpSub&) = delete;
  ZmtpSub& operator=(const ZmtpSub&) = delete;

  // "tcp://host:port"; returns false with a reason in error()
  bool connect(const std::string& endpoint, const std::string& topic, int timeout_ms = 3000);
  // next multipart message; blocks up to timeout_ms (<0: forever).
  // Returns 1 message, 0 timeout, -1 connection lost.
  int recv(std::vector<std::string>* frames, int timeout_ms);
  void close();
  const std::string& error() const { return err_; }

 private:
  bool read_n(char* dst, size_t n, int timeout_ms);
  bool send_frame(const std::string& body, bool command, bool more);
  // one frame; *command / *more from the flags byte
  int read_frame(std::string* body, bool* command, bool* more, int timeout_ms);
  int fd_ = -1;
  std::string err_;
};

}  // namespace ib
