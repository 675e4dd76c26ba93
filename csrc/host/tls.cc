#include "tls.h"

#include <openssl/bio.h>
#include <openssl/ec.h>
#include <openssl/err.h>
#include <openssl/evp.h>
#include <openssl/pem.h>
#include <openssl/rand.h>
#include <openssl/ssl.h>
#include <openssl/x509.h>
#include <openssl/x509v3.h>

#include <fcntl.h>
#include <poll.h>
#include <signal.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cerrno>
#include <chrono>
#include <cstring>
#include <mutex>

#include "common.h"
#include "transport.h"

namespace nexar {

namespace {

std::string ssl_error(const char* what) {
  std::string s = what;
  unsigned long e;
  while ((e = ERR_get_error()) != 0) {
    char buf[256];
    ERR_error_string_n(e, buf, sizeof(buf));
    s += ": ";
    s += buf;
  }
  return s;
}

[[noreturn]] void tls_fail(const char* what) { fail(Err::ConnectionFailed, ssl_error(what)); }

EVP_PKEY* new_p256_key() {
  EVP_PKEY* k = EVP_EC_gen("P-256");
  if (!k) tls_fail("EC key generation failed");
  return k;
}

std::string pem_of_cert(X509* c) {
  BIO* b = BIO_new(BIO_s_mem());
  PEM_write_bio_X509(b, c);
  char* d = nullptr;
  long n = BIO_get_mem_data(b, &d);
  std::string s(d, (size_t)n);
  BIO_free(b);
  return s;
}

std::string pem_of_key(EVP_PKEY* k) {
  BIO* b = BIO_new(BIO_s_mem());
  PEM_write_bio_PrivateKey(b, k, nullptr, nullptr, 0, nullptr, nullptr);
  char* d = nullptr;
  long n = BIO_get_mem_data(b, &d);
  std::string s(d, (size_t)n);
  BIO_free(b);
  return s;
}

void add_ext(X509* cert, X509* issuer, int nid, const char* value) {
  X509V3_CTX ctx;
  X509V3_set_ctx_nodb(&ctx);
  X509V3_set_ctx(&ctx, issuer, cert, nullptr, nullptr, 0);
  X509_EXTENSION* ex = X509V3_EXT_conf_nid(nullptr, &ctx, nid, value);
  if (!ex) tls_fail("certificate extension");
  X509_add_ext(cert, ex, -1);
  X509_EXTENSION_free(ex);
}

X509* new_cert(EVP_PKEY* subject_key, const std::string& cn, X509* issuer, EVP_PKEY* issuer_key, bool ca) {
  X509* c = X509_new();
  X509_set_version(c, 2);
  uint64_t serial = 0;
  RAND_bytes(reinterpret_cast<unsigned char*>(&serial), sizeof(serial));
  ASN1_INTEGER_set_uint64(X509_get_serialNumber(c), serial >> 1);
  X509_gmtime_adj(X509_getm_notBefore(c), -3600);
  X509_gmtime_adj(X509_getm_notAfter(c), 60L * 60 * 24 * 365);
  X509_set_pubkey(c, subject_key);
  X509_NAME* name = X509_get_subject_name(c);
  X509_NAME_add_entry_by_txt(name, "CN", MBSTRING_ASC, reinterpret_cast<const unsigned char*>(cn.c_str()), -1, -1, 0);
  X509* iss = issuer ? issuer : c;
  X509_set_issuer_name(c, X509_get_subject_name(iss));
  if (ca) {
    add_ext(c, iss, NID_basic_constraints, "critical,CA:TRUE");
    add_ext(c, iss, NID_key_usage, "critical,keyCertSign,cRLSign");
  } else {
    add_ext(c, iss, NID_basic_constraints, "critical,CA:FALSE");
    add_ext(c, iss, NID_key_usage, "critical,digitalSignature");
    add_ext(c, iss, NID_ext_key_usage, "serverAuth,clientAuth");
  }
  if (!X509_sign(c, issuer_key ? issuer_key : subject_key, EVP_sha256())) tls_fail("certificate signing");
  return c;
}

// ------------------------------------------------------------------ streams
class PlainStream : public Stream {
 public:
  explicit PlainStream(int fd) : fd_(fd) {}
  ~PlainStream() override { close_fd(fd_); }
  void write_all(const void* p, size_t n) override { nexar::write_all(fd_, p, n); }
  bool read_exact(void* p, size_t n) override { return nexar::read_exact(fd_, p, n); }
  size_t read_some(void* p, size_t n) override { return nexar::read_some(fd_, p, n); }
  void write_pair(const void* a, size_t na, const void* b, size_t nb) override {
    nexar::write_pair(fd_, a, na, b, nb);
  }
  void shutdown() override { ::shutdown(fd_, SHUT_RDWR); }
  int fd() const override { return fd_; }

 private:
  int fd_;
};

bool wait_fd(int fd, short events, int ms) {
  pollfd p{fd, events, 0};
  const int r = ::poll(&p, 1, ms);
  return r > 0;
}

class TlsStream : public Stream {
 public:
  TlsStream(int fd, SSL_CTX* ctx) : fd_(fd), ctx_(ctx) {
    ssl_ = SSL_new(ctx_);
    if (!ssl_) tls_fail("SSL_new");
    SSL_set_fd(ssl_, fd_);
    SSL_set_mode(ssl_, SSL_MODE_ENABLE_PARTIAL_WRITE | SSL_MODE_ACCEPT_MOVING_WRITE_BUFFER);
    const int fl = fcntl(fd_, F_GETFL, 0);
    fcntl(fd_, F_SETFL, fl | O_NONBLOCK);
  }
  ~TlsStream() override {
    {
      std::lock_guard<std::mutex> g(mu_);
      if (ssl_) {
        if (!closed_) SSL_shutdown(ssl_);
        SSL_free(ssl_);
        ssl_ = nullptr;
      }
    }
    SSL_CTX_free(ctx_);
    close_fd(fd_);
  }

  void handshake(bool server, double timeout_s) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
      int r, e;
      {
        std::lock_guard<std::mutex> g(mu_);
        r = server ? SSL_accept(ssl_) : SSL_connect(ssl_);
        e = r == 1 ? SSL_ERROR_NONE : SSL_get_error(ssl_, r);
      }
      if (r == 1) return;
      const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      if (dt > timeout_s) fail(Err::ConnectionFailed, "TLS handshake timed out");
      if (e == SSL_ERROR_WANT_READ) wait_fd(fd_, POLLIN, 50);
      else if (e == SSL_ERROR_WANT_WRITE) wait_fd(fd_, POLLOUT, 50);
      else tls_fail(server ? "TLS accept failed" : "TLS connect failed");
    }
  }

  void write_all(const void* p, size_t n) override {
    const char* c = static_cast<const char*>(p);
    while (n > 0) {
      if (closed_) fail(Err::PeerDisconnected, "TLS stream closed");
      int r, e;
      {
        std::lock_guard<std::mutex> g(mu_);
        const int chunk = (int)std::min<size_t>(n, 1u << 30);
        r = SSL_write(ssl_, c, chunk);
        e = r > 0 ? SSL_ERROR_NONE : SSL_get_error(ssl_, r);
      }
      if (r > 0) {
        c += r;
        n -= (size_t)r;
        continue;
      }
      if (e == SSL_ERROR_WANT_WRITE) wait_fd(fd_, POLLOUT, 50);
      else if (e == SSL_ERROR_WANT_READ) wait_fd(fd_, POLLIN, 50);
      else {
        ERR_clear_error();
        fail(Err::PeerDisconnected, "TLS write failed");
      }
    }
  }

  bool read_exact(void* p, size_t n) override {
    char* c = static_cast<char*>(p);
    while (n > 0) {
      if (closed_) return false;
      int r, e;
      {
        std::lock_guard<std::mutex> g(mu_);
        const int chunk = (int)std::min<size_t>(n, 1u << 30);
        r = SSL_read(ssl_, c, chunk);
        e = r > 0 ? SSL_ERROR_NONE : SSL_get_error(ssl_, r);
      }
      if (r > 0) {
        c += r;
        n -= (size_t)r;
        continue;
      }
      if (e == SSL_ERROR_WANT_READ) {
        wait_fd(fd_, POLLIN, 50);
      } else if (e == SSL_ERROR_WANT_WRITE) {
        wait_fd(fd_, POLLOUT, 50);
      } else {
        ERR_clear_error();
        return false;  // close_notify, reset or protocol error
      }
    }
    return true;
  }

  size_t read_some(void* p, size_t n) override {
    while (true) {
      if (closed_) return 0;
      int r, e;
      {
        std::lock_guard<std::mutex> g(mu_);
        r = SSL_read(ssl_, p, (int)std::min<size_t>(n, 1u << 30));
        e = r > 0 ? SSL_ERROR_NONE : SSL_get_error(ssl_, r);
      }
      if (r > 0) return (size_t)r;
      if (e == SSL_ERROR_WANT_READ) {
        wait_fd(fd_, POLLIN, 50);
      } else if (e == SSL_ERROR_WANT_WRITE) {
        wait_fd(fd_, POLLOUT, 50);
      } else {
        ERR_clear_error();
        return 0;
      }
    }
  }

  // A small frame goes out as one TLS record.
  void write_pair(const void* a, size_t na, const void* b, size_t nb) override {
    if (na + nb <= 16384) {
      uint8_t tmp[16384];
      std::memcpy(tmp, a, na);
      if (nb) std::memcpy(tmp + na, b, nb);
      write_all(tmp, na + nb);
      return;
    }
    write_all(a, na);
    if (nb) write_all(b, nb);
  }

  void shutdown() override {
    closed_ = true;
    ::shutdown(fd_, SHUT_RDWR);
  }
  int fd() const override { return fd_; }
  bool encrypted() const override { return true; }

 private:
  int fd_;
  SSL_CTX* ctx_;
  SSL* ssl_ = nullptr;
  std::mutex mu_;
  std::atomic<bool> closed_{false};
};

// OpenSSL's socket BIO writes with write(), not send(MSG_NOSIGNAL) like the
// plain transport, so a write to a peer that already closed raises SIGPIPE,
// whose default action ends the process. Ignore it, unless the embedding
// program installed its own handler (Python already ignores it).
void ignore_sigpipe_once() {
  static std::once_flag once;
  std::call_once(once, [] {
    struct sigaction cur;
    if (sigaction(SIGPIPE, nullptr, &cur) == 0 && cur.sa_handler == SIG_DFL) {
      struct sigaction sa;
      std::memset(&sa, 0, sizeof(sa));
      sa.sa_handler = SIG_IGN;
      sigaction(SIGPIPE, &sa, nullptr);
    }
  });
}

SSL_CTX* make_ctx(bool server, const TlsIdentity& id, bool verify_peer) {
  ignore_sigpipe_once();
  SSL_CTX* ctx = SSL_CTX_new(server ? TLS_server_method() : TLS_client_method());
  if (!ctx) tls_fail("SSL_CTX_new");
  SSL_CTX_set_min_proto_version(ctx, TLS1_3_VERSION);
  if (!id.cert_pem.empty()) {
    BIO* cb = BIO_new_mem_buf(id.cert_pem.data(), (int)id.cert_pem.size());
    X509* cert = PEM_read_bio_X509(cb, nullptr, nullptr, nullptr);
    BIO_free(cb);
    BIO* kb = BIO_new_mem_buf(id.key_pem.data(), (int)id.key_pem.size());
    EVP_PKEY* key = PEM_read_bio_PrivateKey(kb, nullptr, nullptr, nullptr);
    BIO_free(kb);
    if (!cert || !key || SSL_CTX_use_certificate(ctx, cert) != 1 || SSL_CTX_use_PrivateKey(ctx, key) != 1) {
      X509_free(cert);
      EVP_PKEY_free(key);
      SSL_CTX_free(ctx);
      tls_fail("loading the node certificate");
    }
    X509_free(cert);
    EVP_PKEY_free(key);
  }
  if (verify_peer) {
    X509_STORE* store = SSL_CTX_get_cert_store(ctx);
    BIO* b = BIO_new_mem_buf(id.ca_cert_pem.data(), (int)id.ca_cert_pem.size());
    X509* ca = PEM_read_bio_X509(b, nullptr, nullptr, nullptr);
    BIO_free(b);
    if (!ca || X509_STORE_add_cert(store, ca) != 1) {
      X509_free(ca);
      SSL_CTX_free(ctx);
      tls_fail("loading the cluster CA");
    }
    X509_free(ca);
    SSL_CTX_set_verify(ctx, SSL_VERIFY_PEER | (server ? SSL_VERIFY_FAIL_IF_NO_PEER_CERT : 0), nullptr);
  } else {
    SSL_CTX_set_verify(ctx, SSL_VERIFY_NONE, nullptr);
  }
  return ctx;
}

}  // namespace

// ------------------------------------------------------------------ CA
std::shared_ptr<ClusterCA> ClusterCA::generate(const std::string& name) {
  std::shared_ptr<ClusterCA> ca(new ClusterCA());
  EVP_PKEY* k = new_p256_key();
  X509* c = new_cert(k, name, nullptr, nullptr, true);
  ca->key_ = k;
  ca->cert_ = c;
  ca->ca_pem_ = pem_of_cert(c);
  return ca;
}

std::shared_ptr<ClusterCA> ClusterCA::from_pem(const std::string& key_pem, const std::string& cert_pem) {
  BIO* kb = BIO_new_mem_buf(key_pem.data(), (int)key_pem.size());
  BIO* cb = BIO_new_mem_buf(cert_pem.data(), (int)cert_pem.size());
  EVP_PKEY* k = kb ? PEM_read_bio_PrivateKey(kb, nullptr, nullptr, nullptr) : nullptr;
  X509* c = cb ? PEM_read_bio_X509(cb, nullptr, nullptr, nullptr) : nullptr;
  if (kb) BIO_free(kb);
  if (cb) BIO_free(cb);
  if (!k || !c || X509_check_private_key(c, k) != 1) {
    if (k) EVP_PKEY_free(k);
    if (c) X509_free(c);
    fail(Err::Tls, "ClusterCA::from_pem: unreadable key / certificate or the key does not match");
  }
  std::shared_ptr<ClusterCA> ca(new ClusterCA());
  ca->key_ = k;
  ca->cert_ = c;
  ca->ca_pem_ = pem_of_cert(c);
  return ca;
}

std::string ClusterCA::key_pem() const { return pem_of_key(static_cast<EVP_PKEY*>(key_)); }

ClusterCA::~ClusterCA() {
  X509_free(static_cast<X509*>(cert_));
  EVP_PKEY_free(static_cast<EVP_PKEY*>(key_));
}

TlsIdentity ClusterCA::issue(const std::string& common_name) const {
  EVP_PKEY* k = new_p256_key();
  X509* c = new_cert(k, common_name, static_cast<X509*>(cert_), static_cast<EVP_PKEY*>(key_), false);
  TlsIdentity id{ca_pem_, pem_of_cert(c), pem_of_key(k)};
  X509_free(c);
  EVP_PKEY_free(k);
  return id;
}

// ------------------------------------------------------------------ factories
std::shared_ptr<Stream> plain_stream(int fd) { return std::make_shared<PlainStream>(fd); }

std::shared_ptr<Stream> tls_client(int fd, const TlsIdentity& id, bool verify_peer, double timeout_s) {
  SSL_CTX* ctx;
  try {
    ctx = make_ctx(false, id, verify_peer);
  } catch (...) {
    close_fd(fd);
    throw;
  }
  auto s = std::make_shared<TlsStream>(fd, ctx);
  s->handshake(false, timeout_s);
  return s;
}

std::shared_ptr<Stream> tls_server(int fd, const TlsIdentity& id, bool require_client_cert, double timeout_s) {
  SSL_CTX* ctx;
  try {
    ctx = make_ctx(true, id, require_client_cert);
  } catch (...) {
    close_fd(fd);
    throw;
  }
  auto s = std::make_shared<TlsStream>(fd, ctx);
  s->handshake(true, timeout_s);
  return s;
}

void send_identity(Stream& s, const TlsIdentity& id) {
  Bytes b;
  for (const std::string* f : {&id.ca_cert_pem, &id.cert_pem, &id.key_pem}) {
    put_u32(b, (uint32_t)f->size());
    b.insert(b.end(), f->begin(), f->end());
  }
  s.write_all(b.data(), b.size());
}

TlsIdentity recv_identity(Stream& s) {
  TlsIdentity id;
  for (std::string* f : {&id.ca_cert_pem, &id.cert_pem, &id.key_pem}) {
    uint8_t lb[4];
    if (!s.read_exact(lb, 4)) fail(Err::ConnectionFailed, "bootstrap: connection closed while receiving the TLS identity");
    const uint32_t n = (uint32_t)get_le(lb, 4);
    if (n > (1u << 20)) fail(Err::DecodeFailed, "bootstrap: oversized TLS identity");
    f->resize(n);
    if (n && !s.read_exact(&(*f)[0], n)) fail(Err::ConnectionFailed, "bootstrap: connection closed");
  }
  return id;
}

}  // namespace nexar
