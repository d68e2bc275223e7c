#include "kiwi/p2p/driver.hpp"

#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "kiwi/common.hpp"

namespace kiwi::p2p {

namespace {
template <typename F>
void load(F& fn, const char* name, int version) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    const cudaError_t e =
        cudaGetDriverEntryPointByVersion(name, &p, version, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
        cudaGetLastError();
        throw kiwi::error(std::string("kiwi::p2p: CUDA driver entry point unavailable: ") + name);
    }
    fn = reinterpret_cast<F>(p);
}
}  // namespace

const Driver& driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        load(d.cuMemCreate, "cuMemCreate", 10020);
        load(d.cuMemRelease, "cuMemRelease", 10020);
        load(d.cuMemExportToShareableHandle, "cuMemExportToShareableHandle", 10020);
        load(d.cuMemImportFromShareableHandle, "cuMemImportFromShareableHandle", 10020);
        load(d.cuMemAddressReserve, "cuMemAddressReserve", 10020);
        load(d.cuMemAddressFree, "cuMemAddressFree", 10020);
        load(d.cuMemMap, "cuMemMap", 10020);
        load(d.cuMemUnmap, "cuMemUnmap", 10020);
        load(d.cuMemSetAccess, "cuMemSetAccess", 10020);
        load(d.cuMemGetAllocationGranularity, "cuMemGetAllocationGranularity", 10020);
        load(d.cuMulticastCreate, "cuMulticastCreate", 12010);
        load(d.cuMulticastAddDevice, "cuMulticastAddDevice", 12010);
        load(d.cuMulticastBindMem, "cuMulticastBindMem", 12010);
        load(d.cuMulticastUnbind, "cuMulticastUnbind", 12010);
        load(d.cuMulticastGetGranularity, "cuMulticastGetGranularity", 12010);
        load(d.cuDeviceGetAttribute, "cuDeviceGetAttribute", 2000);
        load(d.cuDeviceGet, "cuDeviceGet", 2000);
        load(d.cuGetErrorString, "cuGetErrorString", 6000);
        load(d.cuCtxGetCurrent, "cuCtxGetCurrent", 4000);
        load(d.cuStreamWriteValue64, "cuStreamWriteValue64", 11070);
        load(d.cuStreamWaitValue64, "cuStreamWaitValue64", 11070);
    });
    return d;
}

void check_cu(CUresult r, const char* what) {
    if (r == CUDA_SUCCESS) return;
    const char* msg = nullptr;
    try {
        driver().cuGetErrorString(r, &msg);
    } catch (...) {
    }
    throw kiwi::error(std::string("kiwi::p2p: ") + what + " failed: " + (msg ? msg : "unknown") +
                      " (" + std::to_string(static_cast<int>(r)) + ")");
}

}  // namespace kiwi::p2p
