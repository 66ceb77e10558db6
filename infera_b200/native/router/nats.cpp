// Core NATS client (see nats.h).
#include "nats.h"

#include <cstdio>

#include <sys/socket.h>
#include <unistd.h>

#include <chrono>
#include <cstdlib>
#include <sstream>

#include "net.h"

namespace ib {

std::map<std::string, std::string> nats_parse_headers(const std::string& block) {
  std::map<std::string, std::string> out;
  std::istringstream in(block);
  std::string line;
  bool first = true;
  while (std::getline(in, line)) {
    if (!line.empty() && line.back() == '\r') line.pop_back();
    if (first) {
      first = false;
      if (line.compare(0, 8, "NATS/1.0") == 0) {
        std::string rest = line.substr(8);
        size_t a = rest.find_first_not_of(' ');
        if (a != std::string::npos) out["status"] = rest.substr(a, rest.find(' ', a) - a);
      }
      continue;
    }
    if (line.empty()) continue;
    size_t c = line.find(':');
    if (c == std::string::npos) continue;
    size_t v = line.find_first_not_of(' ', c + 1);
    out[line.substr(0, c)] = v == std::string::npos ? "" : line.substr(v);
  }
  return out;
}

NatsConn::~NatsConn() {
  alive_ = false;
  if (fd_ >= 0) ::shutdown(fd_, SHUT_RDWR);
  if (th_.joinable()) th_.join();
  if (fd_ >= 0) ::close(fd_);
}

bool NatsConn::connect(const std::string& url, std::string* err) {
  std::string u = url;
  if (u.compare(0, 7, "nats://") == 0) u = u.substr(7);
  size_t c = u.rfind(':');
  std::string host = c == std::string::npos ? u : u.substr(0, c);
  int port = c == std::string::npos ? 4222 : std::atoi(u.c_str() + c + 1);
  fd_ = tcp_connect(host, port, 5000);
  if (fd_ < 0) {
    *err = "cannot connect to NATS at " + url;
    return false;
  }
  set_timeouts(fd_, 5000, 5000);
  Conn conn(fd_);
  std::string line;
  if (!conn.read_line(&line) || line.compare(0, 5, "INFO ") != 0) {
    *err = "not a NATS server at " + url;
    return false;
  }
  {
    // "max_payload":<n> in the INFO object bounds what the reader accepts
    const size_t at = line.find("\"max_payload\"");
    if (at != std::string::npos) {
      const size_t colon = line.find(':', at);
      if (colon != std::string::npos) {
        const unsigned long long mp = std::strtoull(line.c_str() + colon + 1, nullptr, 10);
        if (mp > 0 && mp < max_payload_) max_payload_ = static_cast<size_t>(mp);
      }
    }
  }
  if (!write("CONNECT {\"verbose\":false,\"pedantic\":false,\"headers\":true,\"no_responders\":true,"
             "\"protocol\":1,\"lang\":\"cpp\",\"version\":\"infera-b200\",\"name\":\"infera-b200-router\"}\r\n"
             "PING\r\n")) {
    *err = "NATS handshake write failed";
    return false;
  }
  while (true) {
    if (!conn.read_line(&line)) {
      *err = "NATS handshake: no PONG";
      return false;
    }
    if (line.compare(0, 4, "PONG") == 0) break;
    if (line.compare(0, 4, "-ERR") == 0) {
      *err = "NATS: " + line;
      return false;
    }
  }
  if (conn.buffered() != 0) {
    *err = "NATS handshake: unexpected data";
    return false;
  }
  set_timeouts(fd_, 0, 5000);   // the reader blocks until data or shutdown
  alive_ = true;
  th_ = std::thread(&NatsConn::reader, this);
  return true;
}

bool NatsConn::write(const std::string& s) {
  std::lock_guard<std::mutex> g(wmu_);
  return write_all(fd_, s);
}

int NatsConn::subscribe(const std::string& subject) {
  int sid;
  {
    std::lock_guard<std::mutex> g(qmu_);
    sid = next_sid_++;
    q_[sid];
  }
  write("SUB " + subject + " " + std::to_string(sid) + "\r\n");
  return sid;
}

void NatsConn::unsubscribe(int sid) {
  write("UNSUB " + std::to_string(sid) + "\r\n");
  std::lock_guard<std::mutex> g(qmu_);
  q_.erase(sid);
}

bool NatsConn::publish(const std::string& subject, const std::string& reply, const std::string& data,
                       const std::vector<std::pair<std::string, std::string>>& headers) {
  std::string rp = reply.empty() ? "" : " " + reply;
  if (headers.empty())
    return write("PUB " + subject + rp + " " + std::to_string(data.size()) + "\r\n" + data + "\r\n");
  std::string hb = "NATS/1.0\r\n";
  for (const auto& h : headers) hb += h.first + ": " + h.second + "\r\n";
  hb += "\r\n";
  return write("HPUB " + subject + rp + " " + std::to_string(hb.size()) + " " +
               std::to_string(hb.size() + data.size()) + "\r\n" + hb + data + "\r\n");
}

bool NatsConn::next(int sid, double timeout_s, NatsMsg* out) {
  std::unique_lock<std::mutex> lk(qmu_);
  auto until = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
  while (true) {
    auto it = q_.find(sid);
    if (it == q_.end()) return false;
    if (!it->second.empty()) {
      *out = std::move(it->second.front());
      it->second.pop_front();
      return true;
    }
    if (!alive_) return false;
    if (cv_.wait_until(lk, until) == std::cv_status::timeout) {
      auto it2 = q_.find(sid);
      if (it2 == q_.end() || it2->second.empty()) return false;
    }
  }
}

void NatsConn::reader() {
  Conn conn(fd_);
  std::string line;
  while (alive_ && conn.read_line(&line, 1 << 20)) {
    bool hmsg = line.compare(0, 5, "HMSG ") == 0;
    if (hmsg || line.compare(0, 4, "MSG ") == 0) {
      std::istringstream in(line.substr(hmsg ? 5 : 4));
      std::vector<std::string> parts;
      std::string w;
      while (in >> w) parts.push_back(w);
      size_t need = hmsg ? 4 : 3;
      if (parts.size() < need) break;
      NatsMsg m;
      m.subject = parts[0];
      int sid = std::atoi(parts[1].c_str());
      if (parts.size() == need + 1) m.reply = parts[2];
      size_t total = std::strtoull(parts.back().c_str(), nullptr, 10);
      size_t hl = hmsg ? std::strtoull(parts[parts.size() - 2].c_str(), nullptr, 10) : 0;
      if (total > max_payload_) {
        std::fprintf(stderr, "[ib200_router] NATS message of %zu bytes exceeds max_payload %zu; closing\n", total,
                     max_payload_);
        break;
      }
      std::string block;
      if (!conn.read_exact(total + 2, &block) || hl > total) break;
      block.resize(total);
      if (hmsg) m.headers = nats_parse_headers(block.substr(0, hl));
      m.data = block.substr(hl);
      std::lock_guard<std::mutex> g(qmu_);
      auto it = q_.find(sid);
      if (it != q_.end()) it->second.push_back(std::move(m));
      cv_.notify_all();
    } else if (line.compare(0, 4, "PING") == 0) {
      write("PONG\r\n");
    }
    // PONG, +OK, INFO and -ERR need no action here
  }
  if (alive_) std::fprintf(stderr, "[ib200_router] NATS connection lost\n");
  std::lock_guard<std::mutex> g(qmu_);
  alive_ = false;
  cv_.notify_all();
}

}  // namespace ib
