// File-descriptor exchange between local ranks with SCM_RIGHTS over
// abstract-namespace Unix sockets (no files on disk, nothing to clean up).
#include <poll.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "kiwi/p2p/heap.hpp"

namespace kiwi::p2p {

namespace {

sockaddr_un make_addr(const std::string& name, socklen_t* len) {
    sockaddr_un a{};
    a.sun_family = AF_UNIX;
    const std::string n = std::string(1, '\0') + name;  // abstract namespace
    if (n.size() > sizeof(a.sun_path)) throw kiwi::error("kiwi::p2p: socket name too long");
    std::memcpy(a.sun_path, n.data(), n.size());
    *len = static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + n.size());
    return a;
}

std::string sock_name(const std::string& job, int rank) { return "kiwi." + job + "." + std::to_string(rank); }

void send_fd(int sock, int fd, int32_t tag) {
    msghdr msg{};
    iovec iov{&tag, sizeof(tag)};
    msg.msg_iov = &iov;
    msg.msg_iovlen = 1;
    alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int))] = {0};
    msg.msg_control = ctrl;
    msg.msg_controllen = sizeof(ctrl);
    cmsghdr* c = CMSG_FIRSTHDR(&msg);
    c->cmsg_level = SOL_SOCKET;
    c->cmsg_type = SCM_RIGHTS;
    c->cmsg_len = CMSG_LEN(sizeof(int));
    std::memcpy(CMSG_DATA(c), &fd, sizeof(int));
    if (sendmsg(sock, &msg, 0) < 0) throw kiwi::error("kiwi::p2p: sendmsg(SCM_RIGHTS) failed");
}

int recv_fd(int sock, int32_t* tag) {
    msghdr msg{};
    iovec iov{tag, sizeof(*tag)};
    msg.msg_iov = &iov;
    msg.msg_iovlen = 1;
    alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int))] = {0};
    msg.msg_control = ctrl;
    msg.msg_controllen = sizeof(ctrl);
    if (recvmsg(sock, &msg, 0) <= 0) throw kiwi::error("kiwi::p2p: recvmsg(SCM_RIGHTS) failed");
    cmsghdr* c = CMSG_FIRSTHDR(&msg);
    if (!c || c->cmsg_type != SCM_RIGHTS) throw kiwi::error("kiwi::p2p: no descriptor received");
    int fd = -1;
    std::memcpy(&fd, CMSG_DATA(c), sizeof(int));
    return fd;
}

bool read_all(int s, void* p, size_t n) {
    auto* b = static_cast<uint8_t*>(p);
    while (n) {
        const ssize_t r = read(s, b, n);
        if (r <= 0) return false;
        b += r;
        n -= static_cast<size_t>(r);
    }
    return true;
}

/// Serves `fd` to `clients` connections (each sends its rank first).
class Server {
public:
    Server(const std::string& name, int fd, int clients, double timeout_s)
        : fd_(fd), clients_(clients), timeout_s_(timeout_s) {
        sock_ = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
        if (sock_ < 0) throw kiwi::error("kiwi::p2p: socket() failed");
        socklen_t len;
        sockaddr_un a = make_addr(name, &len);
        if (bind(sock_, reinterpret_cast<sockaddr*>(&a), len) != 0) {
            close(sock_);
            throw kiwi::error("kiwi::p2p: bind(" + name + ") failed (name in use?)");
        }
        if (listen(sock_, 128) != 0) {
            close(sock_);
            throw kiwi::error("kiwi::p2p: listen() failed");
        }
        th_ = std::thread([this] { run(); });
    }
    ~Server() {
        if (th_.joinable()) th_.join();
        if (sock_ >= 0) close(sock_);
    }
    void join() {
        if (th_.joinable()) th_.join();
        if (!error_.empty()) throw kiwi::error(error_);
    }

private:
    void run() {
        const auto end = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s_);
        int served = 0;
        while (served < clients_) {
            const auto left = std::chrono::duration_cast<std::chrono::milliseconds>(end - std::chrono::steady_clock::now());
            if (left.count() <= 0) {
                error_ = "kiwi::p2p: timed out waiting for peers to fetch the heap descriptor";
                return;
            }
            pollfd p{sock_, POLLIN, 0};
            if (poll(&p, 1, static_cast<int>(std::min<long long>(left.count(), 1000))) <= 0) continue;
            const int c = accept4(sock_, nullptr, nullptr, SOCK_CLOEXEC);
            if (c < 0) continue;
            int32_t peer = -1;
            if (read_all(c, &peer, sizeof(peer))) {
                try {
                    send_fd(c, fd_, peer);
                    ++served;
                } catch (const std::exception& e) {
                    error_ = e.what();
                }
            }
            close(c);
        }
    }
    int sock_ = -1;
    int fd_;
    int clients_;
    double timeout_s_;
    std::thread th_;
    std::string error_;
};

int fetch_from(const std::string& name, int32_t my_rank, double timeout_s) {
    const auto end = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
    while (true) {
        const int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
        if (s < 0) throw kiwi::error("kiwi::p2p: socket() failed");
        socklen_t len;
        sockaddr_un a = make_addr(name, &len);
        if (connect(s, reinterpret_cast<sockaddr*>(&a), len) == 0) {
            // Bound the reply wait by what is left of the timeout (a server that
            // accepted but stalled must not block this rank forever).
            const auto left = std::chrono::duration_cast<std::chrono::microseconds>(end - std::chrono::steady_clock::now());
            const long long us = std::max<long long>(left.count(), 1000);
            timeval tv{};
            tv.tv_sec = static_cast<time_t>(us / 1000000);
            tv.tv_usec = static_cast<suseconds_t>(us % 1000000);
            setsockopt(s, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
            if (write(s, &my_rank, sizeof(my_rank)) != sizeof(my_rank)) {
                close(s);
                throw kiwi::error("kiwi::p2p: write to " + name + " failed");
            }
            int32_t tag = -1;
            int fd = -1;
            try {
                fd = recv_fd(s, &tag);
            } catch (...) {
                close(s);
                throw;
            }
            close(s);
            return fd;
        }
        close(s);
        if (std::chrono::steady_clock::now() > end) {
            throw kiwi::error("kiwi::p2p: timed out connecting to " + name);
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(2));
    }
}

}  // namespace

std::vector<int> exchange_fds(const std::string& job, int rank, int world, int my_fd, double timeout_s) {
    if (world < 1 || rank < 0 || rank >= world) throw kiwi::error("kiwi::p2p: bad rank/world");
    std::vector<int> fds(world, -1);
    fds[rank] = dup(my_fd);
    if (world == 1) return fds;
    Server server(sock_name(job, rank), my_fd, world - 1, timeout_s);
    try {
        for (int k = 1; k < world; ++k) {
            const int peer = (rank + k) % world;
            fds[peer] = fetch_from(sock_name(job, peer), rank, timeout_s);
        }
    } catch (...) {
        for (int& f : fds) {
            if (f >= 0) close(f);
        }
        server.join();
        throw;
    }
    server.join();
    return fds;
}

int broadcast_fd(const std::string& job, int rank, int world, int root, int fd, double timeout_s) {
    const std::string name = sock_name(job + ".bcast", root);
    if (rank == root) {
        Server server(name, fd, world - 1, timeout_s);
        server.join();
        return dup(fd);
    }
    return fetch_from(name, rank, timeout_s);
}

}  // namespace kiwi::p2p
