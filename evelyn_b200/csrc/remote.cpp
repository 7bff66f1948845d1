// remote.cpp -- RemoteAarnnFfn: serve chosen FFN layers from AARNN knowledge regions.
//
// Restates src/remote.rs:
//   * one persistent TCP stream per routed layer (Endpoint, :47-53), connect timeout
//     5 s, TCP_NODELAY, read timeout from the constructor, write timeout 30 s (:56-67);
//   * wire format (:69-111): u32 width + width f32 (little endian) out; u32 status,
//     u32 width, width f32 back; status != 0, a width mismatch or a non-finite value is
//     an error;
//   * one reconnect per call (:114-143) and per-endpoint stats (:145-154);
//   * on failure the layer runs the dense FFN and `fallbacks` counts it (:247-271),
//     with the same stderr line.
// The engine calls it through the evl_ffn_backend hook, on the host, only for the
// routed layers; every other layer stays on the device.
#include <arpa/inet.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "engine.hpp"

namespace evl {
namespace {

struct IoError {
    std::string msg;
};

class Endpoint {
public:
    Endpoint(std::string addr, uint32_t timeout_ms) : addr_(std::move(addr)), timeout_ms_(timeout_ms) {}
    ~Endpoint() {
        if (fd_ >= 0) ::close(fd_);
    }

    bool call(const float* x, size_t n, std::vector<float>& y, std::string& err) {
        const auto t0 = std::chrono::steady_clock::now();
        uint64_t attempts = 0;
        bool ok = false;
        {
            std::lock_guard<std::mutex> g(mu_);
            std::string last = "request failed";
            for (int i = 0; i < 2 && !ok; ++i) {
                ++attempts;
                try {
                    if (fd_ < 0) fd_ = connect_();
                } catch (const IoError& e) {
                    last = e.msg;
                    continue;
                }
                try {
                    exchange(x, n, y);
                    ok = true;
                } catch (const IoError& e) {
                    ::close(fd_);
                    fd_ = -1;
                    last = e.msg;
                }
            }
            if (!ok) err = last;
        }
        const uint64_t ns = (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                std::chrono::steady_clock::now() - t0)
                                .count();
        std::lock_guard<std::mutex> g(stats_mu_);
        stats_.calls += 1;
        stats_.retries += attempts - 1;
        stats_.total_ns += ns;
        stats_.max_ns = std::max<uint64_t>(stats_.max_ns, ns);
        if (!ok) stats_.failures += 1;
        return ok;
    }

    evl_endpoint_stats stats() {
        std::lock_guard<std::mutex> g(stats_mu_);
        return stats_;
    }
    const std::string& addr() const { return addr_; }

private:
    int connect_() {
        const size_t colon = addr_.rfind(':');
        if (colon == std::string::npos) throw IoError{"invalid socket address"};
        std::string host = addr_.substr(0, colon), port = addr_.substr(colon + 1);
        if (host.size() > 2 && host.front() == '[' && host.back() == ']') host = host.substr(1, host.size() - 2);
        addrinfo hints{};
        hints.ai_socktype = SOCK_STREAM;
        addrinfo* res = nullptr;
        if (getaddrinfo(host.c_str(), port.c_str(), &hints, &res) != 0 || !res)
            throw IoError{"endpoint resolved to no addresses"};
        int fd = ::socket(res->ai_family, SOCK_STREAM, 0);
        if (fd < 0) {
            freeaddrinfo(res);
            throw IoError{std::string("socket: ") + strerror(errno)};
        }
        const int fl = fcntl(fd, F_GETFL, 0);
        fcntl(fd, F_SETFL, fl | O_NONBLOCK);
        int rc = ::connect(fd, res->ai_addr, res->ai_addrlen);
        freeaddrinfo(res);
        if (rc != 0 && errno != EINPROGRESS) {
            std::string m = strerror(errno);
            ::close(fd);
            throw IoError{m};
        }
        if (rc != 0) {  // connect_timeout 5 s
            pollfd p{fd, POLLOUT, 0};
            rc = ::poll(&p, 1, 5000);
            int soerr = 0;
            socklen_t len = sizeof(soerr);
            getsockopt(fd, SOL_SOCKET, SO_ERROR, &soerr, &len);
            if (rc <= 0 || soerr != 0) {
                ::close(fd);
                throw IoError{rc == 0 ? "connection timed out" : strerror(soerr ? soerr : errno)};
            }
        }
        fcntl(fd, F_SETFL, fl & ~O_NONBLOCK);
        int one = 1;
        setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
        // set_read_timeout(Some(Duration::ZERO)) is an error in the reference (a zero
        // SO_RCVTIMEO would mean "no timeout" here): the connection fails, so the layer
        // falls back to the dense FFN like remote.rs:62-64 does
        if (timeout_ms_ == 0) {
            ::close(fd);
            throw IoError{"cannot set a 0 duration timeout"};
        }
        timeval rt{(time_t)(timeout_ms_ / 1000), (suseconds_t)((timeout_ms_ % 1000) * 1000)};
        setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &rt, sizeof(rt));
        timeval wt{30, 0};
        setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &wt, sizeof(wt));
        return fd;
    }

    void write_all(const void* p, size_t n) {
        const uint8_t* b = static_cast<const uint8_t*>(p);
        while (n) {
            ssize_t w = ::send(fd_, b, n, MSG_NOSIGNAL);
            if (w < 0 && errno == EINTR) continue;  // write_all retries Interrupted
            if (w <= 0) throw IoError{w == 0 ? "write zero" : strerror(errno)};
            b += w;
            n -= (size_t)w;
        }
    }
    void read_exact(void* p, size_t n) {
        uint8_t* b = static_cast<uint8_t*>(p);
        while (n) {
            ssize_t r = ::recv(fd_, b, n, 0);
            if (r < 0 && errno == EINTR) continue;  // read_exact retries Interrupted
            if (r == 0) throw IoError{"failed to fill whole buffer"};
            if (r < 0) throw IoError{strerror(errno)};
            b += r;
            n -= (size_t)r;
        }
    }

    void exchange(const float* x, size_t n, std::vector<float>& y) {
        if (n > 0xffffffffull) throw IoError{"input width exceeds protocol limit"};
        const uint32_t width = (uint32_t)n;
        std::vector<uint8_t> buf(4 + n * 4);
        std::memcpy(buf.data(), &width, 4);  // little-endian host
        std::memcpy(buf.data() + 4, x, n * 4);
        write_all(buf.data(), buf.size());
        uint32_t h[2];
        read_exact(h, 8);
        if (h[0] != 0) throw IoError{"region returned status " + std::to_string(h[0])};
        if (h[1] != width)
            throw IoError{"region returned width " + std::to_string(h[1]) + "; expected " + std::to_string(width)};
        y.resize(h[1]);
        read_exact(y.data(), (size_t)h[1] * 4);
        for (float v : y)
            if (!std::isfinite(v)) throw IoError{"region returned a non-finite value"};
    }

    std::string addr_;
    uint32_t timeout_ms_;
    std::mutex mu_;
    int fd_ = -1;
    std::mutex stats_mu_;
    evl_endpoint_stats stats_{};
};

}  // namespace
}  // namespace evl

struct evl_remote_ffn {
    std::map<size_t, std::unique_ptr<evl::Endpoint>> endpoints;
    std::vector<uint8_t> routed;
    std::atomic<uint64_t> fallbacks{0};
};

namespace {

int remote_ffn_cb(void* ctx, size_t layer, const float* x, size_t n, float* y) {
    auto* r = static_cast<evl_remote_ffn*>(ctx);
    auto it = r->endpoints.find(layer);
    if (it == r->endpoints.end()) return EVL_FFN_DENSE;
    std::vector<float> out;
    std::string err;
    if (it->second->call(x, n, out, err)) {
        if (out.size() == n) {
            std::memcpy(y, out.data(), n * 4);
            return 0;
        }
        std::fprintf(stderr, "aarnn region %s: width %zu != %zu; dense fallback\n", it->second->addr().c_str(),
                     out.size(), n);
    } else {
        std::fprintf(stderr, "aarnn region %s: %s; dense fallback\n", it->second->addr().c_str(), err.c_str());
    }
    r->fallbacks.fetch_add(1);
    return EVL_FFN_DENSE;
}

}  // namespace

extern "C" {

evl_status evl_remote_ffn_new(evl_model* model, size_t n, const size_t* layers, const char* const* addrs,
                              uint32_t timeout_ms, evl_remote_ffn** out) {
    if (!out || (n && (!layers || !addrs))) {
        evl::set_last_error("null argument");
        return EVL_ERR_INVALID_INPUT;
    }
    auto* r = new evl_remote_ffn();
    size_t L = 0;
    if (model) {
        L = model->m->cfg.layers;
    } else {  // no model: size the routing table by the routed layers themselves
        for (size_t i = 0; i < n; ++i) L = std::max(L, layers[i] + 1);
    }
    r->routed.assign(L, 0);
    for (size_t i = 0; i < n; ++i) {
        if (layers[i] >= L || !addrs[i]) {
            evl::set_last_error("routed layer " + std::to_string(layers[i]) + " is outside the model");
            delete r;
            return EVL_ERR_INVALID_INPUT;
        }
        r->endpoints[layers[i]] = std::make_unique<evl::Endpoint>(addrs[i], timeout_ms);
        r->routed[layers[i]] = 1;
    }
    *out = r;
    return EVL_OK;
}

void evl_remote_ffn_free(evl_remote_ffn* r) { delete r; }

evl_status evl_remote_ffn_backend(evl_remote_ffn* r, evl_ffn_backend* out) {
    if (!r || !out) {
        evl::set_last_error("null argument");
        return EVL_ERR_INVALID_INPUT;
    }
    out->ffn = remote_ffn_cb;
    out->ctx = r;
    out->routed = r->routed.data();
    out->routed_len = r->routed.size();
    out->fallbacks = nullptr;  // the region counts its own fallbacks
    return EVL_OK;
}

uint64_t evl_remote_ffn_fallbacks(const evl_remote_ffn* r) { return r ? r->fallbacks.load() : 0; }

evl_status evl_remote_ffn_stats(const evl_remote_ffn* r, size_t layer, evl_endpoint_stats* out) {
    if (!r || !out) {
        evl::set_last_error("null argument");
        return EVL_ERR_INVALID_INPUT;
    }
    auto it = r->endpoints.find(layer);
    if (it == r->endpoints.end()) {
        evl::set_last_error("layer " + std::to_string(layer) + " is not routed");
        return EVL_ERR_NOT_FOUND;
    }
    *out = it->second->stats();
    return EVL_OK;
}

}  // extern "C"
