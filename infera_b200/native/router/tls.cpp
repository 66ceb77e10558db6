// TLS client sessions over a connected socket (see net.h), for the
// Kubernetes API server: peer verification against the given CA bundle (or
// the system store) and the server name / IP checked against the
// certificate.
#include <arpa/inet.h>
#include <openssl/err.h>
#include <openssl/ssl.h>
#include <openssl/x509v3.h>

#include <map>
#include <mutex>

#include "net.h"

namespace ib {

struct TlsSession {
  SSL* ssl = nullptr;
};

namespace {

std::mutex g_mu;
std::map<std::string, SSL_CTX*> g_ctx;  // per CA bundle, kept for the process

SSL_CTX* ctx_for(const std::string& ca_file, std::string* err) {
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_ctx.find(ca_file);
  if (it != g_ctx.end()) return it->second;
  SSL_CTX* ctx = SSL_CTX_new(TLS_client_method());
  if (ctx == nullptr) {
    *err = "SSL_CTX_new failed";
    return nullptr;
  }
  SSL_CTX_set_min_proto_version(ctx, TLS1_2_VERSION);
  SSL_CTX_set_verify(ctx, SSL_VERIFY_PEER, nullptr);
  const int ok = ca_file.empty() ? SSL_CTX_set_default_verify_paths(ctx)
                                 : SSL_CTX_load_verify_locations(ctx, ca_file.c_str(), nullptr);
  if (ok != 1) {
    *err = "cannot load CA bundle " + (ca_file.empty() ? std::string("(system)") : ca_file);
    SSL_CTX_free(ctx);
    return nullptr;
  }
  g_ctx[ca_file] = ctx;
  return ctx;
}

std::string ssl_error() {
  char buf[256];
  const unsigned long e = ERR_get_error();
  if (e == 0) return "TLS error";
  ERR_error_string_n(e, buf, sizeof buf);
  return buf;
}

}  // namespace

TlsSession* tls_connect(int fd, const std::string& host, const std::string& ca_file, std::string* err) {
  SSL_CTX* ctx = ctx_for(ca_file, err);
  if (ctx == nullptr) return nullptr;
  SSL* ssl = SSL_new(ctx);
  if (ssl == nullptr) {
    *err = ssl_error();
    return nullptr;
  }
  SSL_set_fd(ssl, fd);
  X509_VERIFY_PARAM* vp = SSL_get0_param(ssl);
  in6_addr a6;
  in_addr a4;
  const bool is_ip = inet_pton(AF_INET, host.c_str(), &a4) == 1 || inet_pton(AF_INET6, host.c_str(), &a6) == 1;
  if (is_ip) {
    X509_VERIFY_PARAM_set1_ip_asc(vp, host.c_str());
  } else {
    SSL_set_tlsext_host_name(ssl, host.c_str());
    X509_VERIFY_PARAM_set1_host(vp, host.c_str(), 0);
  }
  if (SSL_connect(ssl) != 1) {
    *err = "TLS handshake with " + host + ": " + ssl_error();
    SSL_free(ssl);
    return nullptr;
  }
  auto* s = new TlsSession;
  s->ssl = ssl;
  return s;
}

void tls_free(TlsSession* s) {
  if (s == nullptr) return;
  SSL_shutdown(s->ssl);
  SSL_free(s->ssl);
  delete s;
}

long tls_read(TlsSession* s, char* dst, size_t cap) {
  const int n = SSL_read(s->ssl, dst, static_cast<int>(cap > (1u << 30) ? (1u << 30) : cap));
  if (n > 0) return n;
  const int e = SSL_get_error(s->ssl, n);
  return e == SSL_ERROR_ZERO_RETURN ? 0 : -1;
}

size_t tls_pending(TlsSession* s) { return static_cast<size_t>(SSL_pending(s->ssl)); }

bool tls_write_all(TlsSession* s, const std::string& data) {
  size_t off = 0;
  while (off < data.size()) {
    const int n = SSL_write(s->ssl, data.data() + off, static_cast<int>(data.size() - off));
    if (n <= 0) return false;
    off += static_cast<size_t>(n);
  }
  return true;
}

}  // namespace ib
