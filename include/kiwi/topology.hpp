// CPU affinity for progress/proxy threads: pin them to cores on the GPU's own
// NUMA node, because a cross-socket poller adds ~1-2 us to every round trip.
//
// Parity with the reference's topology helpers
// (apps/common/topology/topology.cpp:88-183 of AMDResearch/kiwi): read the
// GPU's PCI-local CPU list from sysfs, intersect it with the process mask,
// bind threads to it.  NIC selection (topology.cpp:185-469) has no B200
// counterpart: NVLink peers need no NIC.
#pragma once

#include <string>
#include <vector>

namespace kiwi::topology {

/// PCI bus id ("0000:1b:00.0") of a CUDA device, lower case; empty on failure.
std::string pci_bus_id(int device);

/// Parses a sysfs cpulist ("0-3,8,10-11").
std::vector<int> parse_cpulist(const std::string& s);

/// CPUs local to `device` that this process may run on.  Falls back to the
/// whole process mask when sysfs gives nothing.  `sysfs_root` is for tests.
std::vector<int> gpu_local_cpus(int device, const std::string& sysfs_root = "/sys");

/// Cores for `n` busy-polling host threads (progress / proxy threads) that
/// serve `device`: the GPU's local CPUs without core 0 (left to the OS) when
/// there are others, starting at offset device * n.  Processes that drive
/// different GPUs sharing one CPU list (a single-node VM reports the same list
/// for every GPU) then pin their pollers to different cores: two spinning
/// pollers on one core time-share it in scheduler slices of milliseconds.
std::vector<int> poller_cpus(int device, size_t n, const std::string& sysfs_root = "/sys");

/// CPUs in this process's affinity mask.
std::vector<int> process_cpus();

/// CPUs in the calling thread's affinity mask.
std::vector<int> current_thread_cpus();

/// Pins the calling thread to `cpus`; returns false if the kernel refused.
bool bind_current_thread(const std::vector<int>& cpus);

/// NUMA node of a CUDA device (-1 if unknown).
int gpu_numa_node(int device, const std::string& sysfs_root = "/sys");

}  // namespace kiwi::topology
