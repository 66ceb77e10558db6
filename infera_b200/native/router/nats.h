// Core NATS client for the native router's bus request transport.
//
// One TCP connection to a NATS server speaking the public client protocol:
// INFO / CONNECT (headers on) / PING-PONG, SUB / UNSUB, PUB / HPUB with a
// "NATS/1.0" header block, and MSG / HMSG deliveries parsed by a reader
// thread into per-subscription queues that request threads wait on.
// Reference counterpart: the Rust router's NATS transport
// (rust/router/src/nats_request.rs), re-written over this router's sockets.
#pragma once

#include <atomic>
#include <condition_variable>
#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <utility>
#include <vector>

namespace ib {

struct NatsMsg {
  std::string subject, reply, data;
  std::map<std::string, std::string> headers;  // "status" holds a NATS/1.0 status code
};

class NatsConn {
 public:
  ~NatsConn();
  // url: nats://host:port (or host:port)
  bool connect(const std::string& url, std::string* err);
  int subscribe(const std::string& subject);
  void unsubscribe(int sid);
  bool publish(const std::string& subject, const std::string& reply, const std::string& data,
               const std::vector<std::pair<std::string, std::string>>& headers);
  // next message of a subscription; false after timeout_s without one (or on a lost connection)
  bool next(int sid, double timeout_s, NatsMsg* out);
  bool alive() const { return alive_; }
  // largest message the reader accepts (the server's INFO max_payload when it
  // states one, else 64 MiB); a larger one closes the connection
  size_t max_payload() const { return max_payload_; }

 private:
  void reader();
  bool write(const std::string& s);
  int fd_ = -1;
  std::atomic<bool> alive_{false};
  std::thread th_;
  std::mutex wmu_;
  std::mutex qmu_;
  std::condition_variable cv_;
  std::map<int, std::deque<NatsMsg>> q_;
  int next_sid_ = 1;
  size_t max_payload_ = size_t(64) << 20;
};

std::map<std::string, std::string> nats_parse_headers(const std::string& block);

}  // namespace ib
