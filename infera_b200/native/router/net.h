// Sockets and HTTP/1.1 framing for the native router: blocking TCP with
// timeouts, request parsing on the server side, a streaming client for the
// upstream leg (Content-Length, chunked, or read-to-close bodies).
#pragma once

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace ib {

struct Url {
  std::string host;
  int port = 80;
  std::string path;  // with leading '/', may be empty
};
bool parse_url(const std::string& url, Url* out);

int tcp_listen(const std::string& host, int port, int backlog = 1024);
// connect with a timeout (ms); returns fd or -1
int tcp_connect(const std::string& host, int port, int timeout_ms);
void set_timeouts(int fd, int recv_ms, int send_ms);
bool write_all(int fd, const char* p, size_t n);
inline bool write_all(int fd, const std::string& s) { return write_all(fd, s.data(), s.size()); }

// TLS client sessions (OpenSSL) for the Kubernetes API server; the data
// plane itself stays plain HTTP. ca_file empty: the system trust store.
struct TlsSession;
TlsSession* tls_connect(int fd, const std::string& host, const std::string& ca_file, std::string* err);
void tls_free(TlsSession* s);
long tls_read(TlsSession* s, char* dst, size_t cap);  // 0 = closed, -1 = error
size_t tls_pending(TlsSession* s);                     // decrypted bytes ready to read
bool tls_write_all(TlsSession* s, const std::string& data);

std::string base64_encode(const std::string& in);
std::string base64_decode(const std::string& in);
std::string lower(std::string s);

// Buffered reader over a socket.
class Conn {
 public:
  explicit Conn(int fd = -1) : fd_(fd) {}
  int fd() const { return fd_; }
  // read through a TLS session on fd (not owned)
  void set_tls(TlsSession* t) { tls_ = t; }
  void reset(int fd) { fd_ = fd; buf_.clear(); off_ = 0; }
  // read until "\r\n\r\n"; returns the header block (without the blank line)
  bool read_head(std::string* head, size_t max_bytes = 1 << 20);
  bool read_exact(size_t n, std::string* out);
  bool read_line(std::string* line, size_t max_bytes = 1 << 16);  // without CRLF
  // some bytes (buffered first); 0 = orderly close, -1 = error
  long read_some(char* dst, size_t cap);
  size_t buffered() const { return buf_.size() - off_; }

 private:
  bool fill();
  long raw_read(char* dst, size_t cap);
  int fd_;
  TlsSession* tls_ = nullptr;
  std::string buf_;
  size_t off_ = 0;
};

struct HttpRequest {
  std::string method, target, path, query, version;
  std::vector<std::pair<std::string, std::string>> headers;  // names lower-cased
  std::string body;
  bool keep_alive = true;
  const std::string* header(const std::string& lname) const;
};

// Parse one request (head + body) from a client connection.
// Returns 1 ok, 0 closed cleanly before a request, -1 malformed / error.
int read_request(Conn& c, HttpRequest* req, size_t max_body = 256u << 20);

struct HttpResponseHead {
  int status = 0;
  std::vector<std::pair<std::string, std::string>> headers;
  bool chunked = false;
  long long content_length = -1;
  bool keep_alive = true;
  const std::string* header(const std::string& lname) const;
};

// Upstream body reader: yields decoded body bytes in pieces.
class BodyReader {
 public:
  BodyReader(Conn& c, const HttpResponseHead& h) : c_(c), chunked_(h.chunked), left_(h.content_length) {}
  // appends the next piece to *out; returns false at the end of the body
  // (check error() to tell a clean end from a broken one)
  bool next(std::string* out);
  bool error() const { return err_; }
  bool complete() const { return done_ && !err_; }

 private:
  Conn& c_;
  bool chunked_;
  long long left_;
  long long chunk_left_ = 0;
  bool done_ = false, err_ = false;
};

bool read_response_head(Conn& c, HttpResponseHead* h);

const char* status_text(int code);
std::string response_head(int status, const std::string& content_type, long long content_length,
                          const std::vector<std::pair<std::string, std::string>>& extra, bool keep_alive);
bool send_simple(int fd, int status, const std::string& content_type, const std::string& body,
                 const std::vector<std::pair<std::string, std::string>>& extra = {}, bool keep_alive = true);
bool send_chunk(int fd, const char* p, size_t n);
bool send_last_chunk(int fd);

}  // namespace ib
