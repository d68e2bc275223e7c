#include "kiwi/topology.hpp"

#include <cuda_runtime.h>
#include <pthread.h>
#include <sched.h>

#include <algorithm>
#include <cctype>
#include <fstream>
#include <sstream>

namespace kiwi::topology {

std::string pci_bus_id(int device) {
    char buf[64] = {0};
    if (cudaDeviceGetPCIBusId(buf, sizeof(buf), device) != cudaSuccess) {
        cudaGetLastError();
        return {};
    }
    std::string s(buf);
    std::transform(s.begin(), s.end(), s.begin(), [](unsigned char c) { return std::tolower(c); });
    // CUDA reports an 8-digit domain ("00000000:1b:00.0"); sysfs uses 4.
    const auto colon = s.find(':');
    if (colon != std::string::npos && colon > 4) s = s.substr(colon - 4);
    return s;
}

std::vector<int> parse_cpulist(const std::string& s) {
    std::vector<int> out;
    std::stringstream ss(s);
    std::string part;
    while (std::getline(ss, part, ',')) {
        part.erase(std::remove_if(part.begin(), part.end(), [](unsigned char c) { return std::isspace(c); }),
                   part.end());
        if (part.empty()) continue;
        const auto dash = part.find('-');
        try {
            if (dash == std::string::npos) {
                out.push_back(std::stoi(part));
            } else {
                const int a = std::stoi(part.substr(0, dash));
                const int b = std::stoi(part.substr(dash + 1));
                for (int c = a; c <= b; ++c) out.push_back(c);
            }
        } catch (...) {
            return {};
        }
    }
    return out;
}

std::vector<int> process_cpus() {
    std::vector<int> out;
    cpu_set_t set;
    CPU_ZERO(&set);
    if (sched_getaffinity(0, sizeof(set), &set) != 0) return out;
    for (int c = 0; c < CPU_SETSIZE; ++c) {
        if (CPU_ISSET(c, &set)) out.push_back(c);
    }
    return out;
}

static std::string read_first_line(const std::string& path) {
    std::ifstream f(path);
    std::string line;
    if (f) std::getline(f, line);
    return line;
}

std::vector<int> gpu_local_cpus(int device, const std::string& sysfs_root) {
    const std::vector<int> allowed = process_cpus();
    const std::string bdf = pci_bus_id(device);
    if (bdf.empty()) return allowed;
    const std::vector<int> local =
        parse_cpulist(read_first_line(sysfs_root + "/bus/pci/devices/" + bdf + "/local_cpulist"));
    std::vector<int> out;
    for (int c : local) {
        if (std::find(allowed.begin(), allowed.end(), c) != allowed.end()) out.push_back(c);
    }
    return out.empty() ? allowed : out;
}

std::vector<int> poller_cpus(int device, size_t n, const std::string& sysfs_root) {
    std::vector<int> local = gpu_local_cpus(device, sysfs_root);
    if (local.size() > 1 && local.front() == 0) local.erase(local.begin());
    std::vector<int> out;
    if (local.empty() || n == 0) return out;
    const size_t start = (static_cast<size_t>(device < 0 ? 0 : device) * n) % local.size();
    for (size_t t = 0; t < n; ++t) out.push_back(local[(start + t) % local.size()]);
    return out;
}

std::vector<int> current_thread_cpus() {
    std::vector<int> out;
    cpu_set_t set;
    CPU_ZERO(&set);
    if (pthread_getaffinity_np(pthread_self(), sizeof(set), &set) != 0) return out;
    for (int c = 0; c < CPU_SETSIZE; ++c) {
        if (CPU_ISSET(c, &set)) out.push_back(c);
    }
    return out;
}

bool bind_current_thread(const std::vector<int>& cpus) {
    if (cpus.empty()) return false;
    cpu_set_t set;
    CPU_ZERO(&set);
    for (int c : cpus) {
        if (c >= 0 && c < CPU_SETSIZE) CPU_SET(c, &set);
    }
    return pthread_setaffinity_np(pthread_self(), sizeof(set), &set) == 0;
}

int gpu_numa_node(int device, const std::string& sysfs_root) {
    const std::string bdf = pci_bus_id(device);
    if (bdf.empty()) return -1;
    const std::string s = read_first_line(sysfs_root + "/bus/pci/devices/" + bdf + "/numa_node");
    try {
        return s.empty() ? -1 : std::stoi(s);
    } catch (...) {
        return -1;
    }
}

}  // namespace kiwi::topology
