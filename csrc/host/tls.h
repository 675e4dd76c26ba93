// TLS 1.3 for the host transport: a per-cluster certificate authority and
// mutually authenticated connections (OpenSSL).
//
// Trust model (as nexar/src/transport/tls.rs:9-173): the seed generates an
// ephemeral cluster CA and issues every node a leaf certificate for it. The
// bootstrap link (worker -> seed) is TLS without certificate verification on
// the worker side and is authenticated by the cluster token; over it the seed
// hands the worker its key, its certificate and the CA certificate. Every
// mesh link afterwards verifies the peer's certificate against the cluster CA
// in both directions.
//
// Streams: the transport reads a connection on one thread (its router) while
// any number of threads write to it. A TLS stream therefore puts the socket in
// non-blocking mode and serialises every OpenSSL call on the connection with a
// mutex that is never held while waiting (poll runs unlocked).
#pragma once
#include <memory>
#include <string>

namespace nexar {

struct TlsIdentity {
  std::string ca_cert_pem;  // cluster CA certificate (trust root)
  std::string cert_pem;     // this node's certificate, signed by the CA
  std::string key_pem;      // this node's private key
  bool valid() const { return !ca_cert_pem.empty() && !cert_pem.empty() && !key_pem.empty(); }
};

class ClusterCA {
 public:
  // New P-256 key and self-signed CA certificate.
  static std::shared_ptr<ClusterCA> generate(const std::string& name = "nexar-cluster-ca");
  ~ClusterCA();
  // Restore a CA saved with key_pem() / cert_pem() (certificate rotation
  // without re-trusting: nexar/src/transport/tls.rs:122-143 persists the CA
  // key pair the same way). Throws if the key does not match the certificate.
  static std::shared_ptr<ClusterCA> from_pem(const std::string& key_pem, const std::string& cert_pem);
  // New P-256 key and a leaf certificate signed by this CA (CN = common_name).
  TlsIdentity issue(const std::string& common_name) const;
  const std::string& cert_pem() const { return ca_pem_; }
  // The CA's private key, PKCS#8 PEM (unencrypted: store it with file
  // permissions that only the operator can read).
  std::string key_pem() const;

 private:
  ClusterCA() = default;
  void* key_ = nullptr;   // EVP_PKEY*
  void* cert_ = nullptr;  // X509*
  std::string ca_pem_;
};

// Byte stream over a connected socket.
class Stream {
 public:
  virtual ~Stream() = default;
  virtual void write_all(const void* p, size_t n) = 0;  // throws NexarError(PeerDisconnected)
  virtual bool read_exact(void* p, size_t n) = 0;       // false on EOF / error
  // Up to n bytes (at least one); 0 on EOF / error.
  virtual size_t read_some(void* p, size_t n) = 0;
  // Two buffers back to back (a frame header and its payload).
  virtual void write_pair(const void* a, size_t na, const void* b, size_t nb) {
    write_all(a, na);
    if (nb) write_all(b, nb);
  }
  virtual void shutdown() = 0;                          // wakes a blocked reader
  virtual int fd() const = 0;
  virtual bool encrypted() const { return false; }
};

std::shared_ptr<Stream> plain_stream(int fd);
// TLS client / server handshake over `fd` (takes ownership). With verify,
// the peer must present a certificate signed by id.ca_cert_pem. The server
// always presents id's certificate; a client presents it when id is valid.
std::shared_ptr<Stream> tls_client(int fd, const TlsIdentity& id, bool verify_peer, double timeout_s);
std::shared_ptr<Stream> tls_server(int fd, const TlsIdentity& id, bool require_client_cert, double timeout_s);

// Length-prefixed transfer of an identity over a stream (bootstrap only).
void send_identity(Stream& s, const TlsIdentity& id);
TlsIdentity recv_identity(Stream& s);

}  // namespace nexar
