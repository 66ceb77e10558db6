// Sockets and HTTP/1.1 framing (see net.h).
#include "net.h"

#include <arpa/inet.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstring>

namespace ib {

std::string lower(std::string s) {
  for (auto& c : s)
    if (c >= 'A' && c <= 'Z') c = static_cast<char>(c - 'A' + 'a');
  return s;
}

bool parse_url(const std::string& url, Url* out) {
  std::string rest = url;
  auto sch = rest.find("://");
  int dflt = 80;
  if (sch != std::string::npos) {
    std::string scheme = lower(rest.substr(0, sch));
    if (scheme == "https") return false;  // no TLS on the data plane
    if (scheme == "tcp") dflt = 0;
    rest = rest.substr(sch + 3);
  }
  auto slash = rest.find('/');
  std::string hostport = slash == std::string::npos ? rest : rest.substr(0, slash);
  out->path = slash == std::string::npos ? "" : rest.substr(slash);
  auto colon = hostport.rfind(':');
  if (colon != std::string::npos && hostport.find(']') == std::string::npos) {
    out->host = hostport.substr(0, colon);
    out->port = std::atoi(hostport.c_str() + colon + 1);
  } else {
    out->host = hostport;
    out->port = dflt;
  }
  if (out->host == "*" || out->host.empty()) out->host = "127.0.0.1";
  return out->port > 0;
}

int tcp_listen(const std::string& host, int port, int backlog) {
  int fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (fd < 0) return -1;
  int one = 1;
  setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_port = htons(static_cast<uint16_t>(port));
  if (host.empty() || host == "0.0.0.0") a.sin_addr.s_addr = INADDR_ANY;
  else if (inet_pton(AF_INET, host.c_str(), &a.sin_addr) != 1) {
    addrinfo hints{}, *res = nullptr;
    hints.ai_family = AF_INET;
    if (getaddrinfo(host.c_str(), nullptr, &hints, &res) != 0 || !res) { ::close(fd); return -1; }
    a.sin_addr = reinterpret_cast<sockaddr_in*>(res->ai_addr)->sin_addr;
    freeaddrinfo(res);
  }
  if (::bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0 || ::listen(fd, backlog) != 0) {
    ::close(fd);
    return -1;
  }
  return fd;
}

int tcp_connect(const std::string& host, int port, int timeout_ms) {
  addrinfo hints{}, *res = nullptr;
  hints.ai_family = AF_UNSPEC;
  hints.ai_socktype = SOCK_STREAM;
  char ps[16];
  std::snprintf(ps, sizeof(ps), "%d", port);
  if (getaddrinfo(host.c_str(), ps, &hints, &res) != 0 || !res) return -1;
  int fd = -1;
  for (addrinfo* ai = res; ai; ai = ai->ai_next) {
    fd = ::socket(ai->ai_family, ai->ai_socktype | SOCK_CLOEXEC | SOCK_NONBLOCK, ai->ai_protocol);
    if (fd < 0) continue;
    int rc = ::connect(fd, ai->ai_addr, ai->ai_addrlen);
    if (rc != 0 && errno == EINPROGRESS) {
      pollfd pf{fd, POLLOUT, 0};
      rc = ::poll(&pf, 1, timeout_ms) == 1 ? 0 : -1;
      if (rc == 0) {
        int e = 0;
        socklen_t l = sizeof(e);
        getsockopt(fd, SOL_SOCKET, SO_ERROR, &e, &l);
        rc = e == 0 ? 0 : -1;
      }
    }
    if (rc == 0) break;
    ::close(fd);
    fd = -1;
  }
  freeaddrinfo(res);
  if (fd >= 0) {
    int fl = fcntl(fd, F_GETFL, 0);
    fcntl(fd, F_SETFL, fl & ~O_NONBLOCK);
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  }
  return fd;
}

void set_timeouts(int fd, int recv_ms, int send_ms) {
  timeval tv{};
  tv.tv_sec = recv_ms / 1000;
  tv.tv_usec = (recv_ms % 1000) * 1000;
  setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
  tv.tv_sec = send_ms / 1000;
  tv.tv_usec = (send_ms % 1000) * 1000;
  setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &tv, sizeof(tv));
}

bool write_all(int fd, const char* p, size_t n) {
  while (n > 0) {
    ssize_t w = ::send(fd, p, n, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    p += w;
    n -= static_cast<size_t>(w);
  }
  return true;
}

static const char kB64[] = "ABCDEFGHIJKLMNOPQRSTUVWXYZabcdefghijklmnopqrstuvwxyz0123456789+/";

std::string base64_encode(const std::string& in) {
  std::string out;
  out.reserve((in.size() + 2) / 3 * 4);
  size_t i = 0;
  const auto* s = reinterpret_cast<const unsigned char*>(in.data());
  for (; i + 2 < in.size(); i += 3) {
    uint32_t v = (s[i] << 16) | (s[i + 1] << 8) | s[i + 2];
    out += kB64[(v >> 18) & 63];
    out += kB64[(v >> 12) & 63];
    out += kB64[(v >> 6) & 63];
    out += kB64[v & 63];
  }
  if (i < in.size()) {
    uint32_t v = s[i] << 16;
    if (i + 1 < in.size()) v |= s[i + 1] << 8;
    out += kB64[(v >> 18) & 63];
    out += kB64[(v >> 12) & 63];
    out += i + 1 < in.size() ? kB64[(v >> 6) & 63] : '=';
    out += '=';
  }
  return out;
}

std::string base64_decode(const std::string& in) {
  int map[256];
  for (int& m : map) m = -1;
  for (int k = 0; k < 64; ++k) map[static_cast<unsigned char>(kB64[k])] = k;
  map[static_cast<unsigned char>('-')] = 62;  // url-safe variants
  map[static_cast<unsigned char>('_')] = 63;
  std::string out;
  uint32_t acc = 0;
  int bits = 0;
  for (unsigned char c : in) {
    int v = map[c];
    if (v < 0) continue;
    acc = (acc << 6) | static_cast<uint32_t>(v);
    bits += 6;
    if (bits >= 8) {
      bits -= 8;
      out.push_back(static_cast<char>((acc >> bits) & 0xFF));
    }
  }
  return out;
}

// ---------------------------------------------------------------------------
// Conn

bool Conn::fill() {
  if (off_ > 0 && off_ == buf_.size()) {
    buf_.clear();
    off_ = 0;
  } else if (off_ > (1 << 16)) {
    buf_.erase(0, off_);
    off_ = 0;
  }
  char tmp[65536];
  while (true) {
    const long r = raw_read(tmp, sizeof(tmp));
    if (r <= 0) return false;
    buf_.append(tmp, static_cast<size_t>(r));
    return true;
  }
}

bool Conn::read_head(std::string* head, size_t max_bytes) {
  // bytes after off_ already searched; relative, because fill() may move
  // the unread bytes to the front of the buffer
  size_t scanned = 0;
  while (true) {
    size_t from = off_ + (scanned > 3 ? scanned - 3 : 0);
    size_t pos = buf_.find("\r\n\r\n", from);
    if (pos != std::string::npos) {
      head->assign(buf_, off_, pos - off_);
      off_ = pos + 4;
      return true;
    }
    if (buf_.size() - off_ > max_bytes) return false;
    scanned = buf_.size() - off_;
    if (!fill()) return false;
  }
}

bool Conn::read_line(std::string* line, size_t max_bytes) {
  while (true) {
    size_t pos = buf_.find("\r\n", off_);
    if (pos != std::string::npos) {
      line->assign(buf_, off_, pos - off_);
      off_ = pos + 2;
      return true;
    }
    if (buf_.size() - off_ > max_bytes) return false;
    if (!fill()) return false;
  }
}

bool Conn::read_exact(size_t n, std::string* out) {
  while (buf_.size() - off_ < n)
    if (!fill()) return false;
  out->append(buf_, off_, n);
  off_ += n;
  return true;
}

long Conn::raw_read(char* dst, size_t cap) {
  if (tls_ != nullptr) return tls_read(tls_, dst, cap);
  ssize_t r;
  do {
    r = ::recv(fd_, dst, cap, 0);
  } while (r < 0 && errno == EINTR);
  return r < 0 ? -1 : static_cast<long>(r);
}

long Conn::read_some(char* dst, size_t cap) {
  if (buffered() == 0) {
    buf_.clear();
    off_ = 0;
    return raw_read(dst, cap);
  }
  size_t n = std::min(cap, buffered());
  std::memcpy(dst, buf_.data() + off_, n);
  off_ += n;
  return static_cast<long>(n);
}

// ---------------------------------------------------------------------------
// HTTP

static void parse_headers(const std::string& head, size_t start,
                          std::vector<std::pair<std::string, std::string>>* out) {
  size_t p = start;
  while (p < head.size()) {
    size_t e = head.find("\r\n", p);
    if (e == std::string::npos) e = head.size();
    size_t colon = head.find(':', p);
    if (colon != std::string::npos && colon < e) {
      std::string name = lower(head.substr(p, colon - p));
      size_t v = colon + 1;
      while (v < e && (head[v] == ' ' || head[v] == '\t')) ++v;
      size_t ve = e;
      while (ve > v && (head[ve - 1] == ' ' || head[ve - 1] == '\t')) --ve;
      out->emplace_back(std::move(name), head.substr(v, ve - v));
    }
    p = e + 2;
  }
}

const std::string* HttpRequest::header(const std::string& lname) const {
  for (const auto& h : headers)
    if (h.first == lname) return &h.second;
  return nullptr;
}

const std::string* HttpResponseHead::header(const std::string& lname) const {
  for (const auto& h : headers)
    if (h.first == lname) return &h.second;
  return nullptr;
}

static bool read_chunked(Conn& c, std::string* body, size_t max_body) {
  while (true) {
    std::string line;
    if (!c.read_line(&line)) return false;
    size_t n = std::strtoul(line.c_str(), nullptr, 16);
    if (n == 0) {
      // trailers until the blank line
      while (true) {
        if (!c.read_line(&line)) return false;
        if (line.empty()) return true;
      }
    }
    if (body->size() + n > max_body) return false;
    if (!c.read_exact(n, body)) return false;
    if (!c.read_line(&line)) return false;
  }
}

int read_request(Conn& c, HttpRequest* req, size_t max_body) {
  std::string head;
  if (!c.read_head(&head)) return c.buffered() == 0 ? 0 : -1;
  size_t e = head.find("\r\n");
  std::string first = head.substr(0, e);
  size_t s1 = first.find(' '), s2 = first.rfind(' ');
  if (s1 == std::string::npos || s2 == s1) return -1;
  req->method = first.substr(0, s1);
  req->target = first.substr(s1 + 1, s2 - s1 - 1);
  req->version = first.substr(s2 + 1);
  auto q = req->target.find('?');
  req->path = q == std::string::npos ? req->target : req->target.substr(0, q);
  req->query = q == std::string::npos ? "" : req->target.substr(q + 1);
  req->headers.clear();
  if (e != std::string::npos) parse_headers(head, e + 2, &req->headers);
  req->keep_alive = req->version != "HTTP/1.0";
  if (const auto* cn = req->header("connection")) {
    std::string v = lower(*cn);
    if (v.find("close") != std::string::npos) req->keep_alive = false;
    if (v.find("keep-alive") != std::string::npos) req->keep_alive = true;
  }
  req->body.clear();
  const auto* te = req->header("transfer-encoding");
  if (te && lower(*te).find("chunked") != std::string::npos) {
    if (!read_chunked(c, &req->body, max_body)) return -1;
  } else if (const auto* cl = req->header("content-length")) {
    size_t n = std::strtoull(cl->c_str(), nullptr, 10);
    if (n > max_body) return -1;
    if (n && !c.read_exact(n, &req->body)) return -1;
  }
  return 1;
}

bool read_response_head(Conn& c, HttpResponseHead* h) {
  std::string head;
  if (!c.read_head(&head)) return false;
  size_t e = head.find("\r\n");
  std::string first = head.substr(0, e);
  size_t s1 = first.find(' ');
  if (s1 == std::string::npos) return false;
  h->status = std::atoi(first.c_str() + s1 + 1);
  h->headers.clear();
  if (e != std::string::npos) parse_headers(head, e + 2, &h->headers);
  h->keep_alive = first.compare(0, 8, "HTTP/1.0") != 0;
  if (const auto* cn = h->header("connection"))
    if (lower(*cn).find("close") != std::string::npos) h->keep_alive = false;
  const auto* te = h->header("transfer-encoding");
  h->chunked = te && lower(*te).find("chunked") != std::string::npos;
  h->content_length = -1;
  if (!h->chunked)
    if (const auto* cl = h->header("content-length")) h->content_length = std::strtoll(cl->c_str(), nullptr, 10);
  return h->status > 0;
}

bool BodyReader::next(std::string* out) {
  if (done_) return false;
  char tmp[65536];
  if (chunked_) {
    if (chunk_left_ == 0) {
      std::string line;
      if (!c_.read_line(&line)) { err_ = done_ = true; return false; }
      if (line.empty() && !c_.read_line(&line)) { err_ = done_ = true; return false; }
      chunk_left_ = static_cast<long long>(std::strtoull(line.c_str(), nullptr, 16));
      if (chunk_left_ == 0) {
        while (true) {  // trailers
          if (!c_.read_line(&line)) { err_ = true; break; }
          if (line.empty()) break;
        }
        done_ = true;
        return false;
      }
    }
    long r = c_.read_some(tmp, static_cast<size_t>(std::min<long long>(chunk_left_, sizeof(tmp))));
    if (r <= 0) { err_ = done_ = true; return false; }
    out->append(tmp, static_cast<size_t>(r));
    chunk_left_ -= r;
    if (chunk_left_ == 0) {
      std::string crlf;
      if (!c_.read_line(&crlf)) { err_ = done_ = true; return false; }
    }
    return true;
  }
  if (left_ == 0) { done_ = true; return false; }
  size_t cap = left_ > 0 ? static_cast<size_t>(std::min<long long>(left_, sizeof(tmp))) : sizeof(tmp);
  long r = c_.read_some(tmp, cap);
  if (r < 0) { err_ = done_ = true; return false; }
  if (r == 0) {
    done_ = true;
    if (left_ > 0) err_ = true;  // closed before Content-Length bytes arrived
    return false;
  }
  out->append(tmp, static_cast<size_t>(r));
  if (left_ > 0) left_ -= r;
  return true;
}

const char* status_text(int code) {
  switch (code) {
    case 200: return "OK";
    case 202: return "Accepted";
    case 204: return "No Content";
    case 400: return "Bad Request";
    case 403: return "Forbidden";
    case 404: return "Not Found";
    case 405: return "Method Not Allowed";
    case 409: return "Conflict";
    case 413: return "Payload Too Large";
    case 429: return "Too Many Requests";
    case 500: return "Internal Server Error";
    case 502: return "Bad Gateway";
    case 503: return "Service Unavailable";
    case 504: return "Gateway Timeout";
    default: return "Status";
  }
}

std::string response_head(int status, const std::string& content_type, long long content_length,
                          const std::vector<std::pair<std::string, std::string>>& extra, bool keep_alive) {
  std::string h;
  char buf[96];
  std::snprintf(buf, sizeof(buf), "HTTP/1.1 %d %s\r\n", status, status_text(status));
  h += buf;
  if (!content_type.empty()) h += "Content-Type: " + content_type + "\r\n";
  if (content_length >= 0) {
    std::snprintf(buf, sizeof(buf), "Content-Length: %lld\r\n", content_length);
    h += buf;
  } else {
    h += "Transfer-Encoding: chunked\r\n";
  }
  for (const auto& kv : extra) h += kv.first + ": " + kv.second + "\r\n";
  h += keep_alive ? "Connection: keep-alive\r\n\r\n" : "Connection: close\r\n\r\n";
  return h;
}

bool send_simple(int fd, int status, const std::string& content_type, const std::string& body,
                 const std::vector<std::pair<std::string, std::string>>& extra, bool keep_alive) {
  std::string out = response_head(status, content_type, static_cast<long long>(body.size()), extra, keep_alive);
  out += body;
  return write_all(fd, out);
}

bool send_chunk(int fd, const char* p, size_t n) {
  if (n == 0) return true;
  char hdr[24];
  int hl = std::snprintf(hdr, sizeof(hdr), "%zx\r\n", n);
  std::string out;
  out.reserve(n + hl + 2);
  out.append(hdr, static_cast<size_t>(hl));
  out.append(p, n);
  out += "\r\n";
  return write_all(fd, out);
}

bool send_last_chunk(int fd) { return write_all(fd, "0\r\n\r\n", 5); }

}  // namespace ib
