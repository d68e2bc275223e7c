#include "kiwi/p2p/heap.hpp"

#include <cuda_runtime.h>
#include <unistd.h>

#include "kiwi/p2p/driver.hpp"

namespace kiwi::p2p {

namespace {
CUdevice cu_device(int device) {
    CUdevice d = 0;
    check_cu(driver().cuDeviceGet(&d, device), "cuDeviceGet");
    return d;
}

CUmemAllocationProp alloc_prop(int device) {
    CUmemAllocationProp p{};
    p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    p.location.id = device;
    p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    return p;
}
}  // namespace

bool SymmetricHeap::multicast_supported(int device) {
    int v = 0;
    try {
        check_cu(driver().cuDeviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, cu_device(device)),
                 "cuDeviceGetAttribute(MULTICAST_SUPPORTED)");
    } catch (...) {
        return false;
    }
    return v != 0;
}

void SymmetricHeap::map_range(CUmemGenericAllocationHandle h, void** va) {
    const Driver& d = driver();
    CUdeviceptr p = 0;
    check_cu(d.cuMemAddressReserve(&p, view_.size, granularity_, 0, 0), "cuMemAddressReserve");
    check_cu(d.cuMemMap(p, view_.size, 0, h, 0), "cuMemMap");
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = device_;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    check_cu(d.cuMemSetAccess(p, view_.size, &acc, 1), "cuMemSetAccess");
    *va = reinterpret_cast<void*>(p);
}

SymmetricHeap::SymmetricHeap(int device, size_t bytes, int rank, int world, const std::string& job,
                             bool multicast, Barrier barrier)
    : device_(device) {
    if (world > kMaxRanks) throw kiwi::error("kiwi::p2p: at most 16 ranks");
    KIWI_CUDA_CHECK(cudaSetDevice(device));
    KIWI_CUDA_CHECK(cudaFree(nullptr));  // make the primary context current
    const Driver& d = driver();
    CUmemAllocationProp prop = alloc_prop(device);
    check_cu(d.cuMemGetAllocationGranularity(&granularity_, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED),
             "cuMemGetAllocationGranularity");
    size_t mc_gran = 0;
    CUmulticastObjectProp mprop{};
    if (multicast) {
        mprop.numDevices = static_cast<unsigned>(world);
        mprop.size = bytes;
        mprop.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
        check_cu(d.cuMulticastGetGranularity(&mc_gran, &mprop, CU_MULTICAST_GRANULARITY_RECOMMENDED),
                 "cuMulticastGetGranularity");
        if (mc_gran > granularity_) granularity_ = mc_gran;
    }
    view_.size = round_up(bytes == 0 ? 1 : bytes, granularity_);
    view_.rank = rank;
    view_.world = world;

    check_cu(d.cuMemCreate(&local_handle_, view_.size, &prop, 0), "cuMemCreate");
    // From here on every acquired resource is released by release() if a later
    // step throws (the destructor does not run for a constructor that threw).
    std::vector<int> fds;
    try {
        int my_fd = -1;
        check_cu(d.cuMemExportToShareableHandle(&my_fd, local_handle_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
                 "cuMemExportToShareableHandle");
        try {
            fds = exchange_fds(job, rank, world, my_fd);
        } catch (...) {
            close(my_fd);
            throw;
        }
        close(my_fd);
        handles_.assign(world, 0);
        for (int r = 0; r < world; ++r) {
            if (r == rank) {
                handles_[r] = local_handle_;
            } else {
                check_cu(d.cuMemImportFromShareableHandle(&handles_[r],
                                                          reinterpret_cast<void*>(static_cast<uintptr_t>(fds[r])),
                                                          CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
                         "cuMemImportFromShareableHandle");
            }
            close(fds[r]);
            fds[r] = -1;
            void* va = nullptr;
            map_range(handles_[r], &va);
            view_.base[r] = static_cast<uint8_t*>(va);
        }
        KIWI_CUDA_CHECK(cudaMemset(view_.base[rank], 0, view_.size));
        KIWI_CUDA_CHECK(cudaDeviceSynchronize());

        if (multicast) {
            mprop.size = view_.size;
            int mc_fd = -1;
            if (rank == 0) {
                check_cu(d.cuMulticastCreate(&mc_handle_, &mprop), "cuMulticastCreate");
                check_cu(d.cuMemExportToShareableHandle(&mc_fd, mc_handle_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR,
                                                        0),
                         "cuMemExportToShareableHandle(multicast)");
            }
            int got = -1;
            try {
                got = broadcast_fd(job, rank, world, 0, mc_fd);
            } catch (...) {
                if (mc_fd >= 0) close(mc_fd);
                throw;
            }
            if (mc_fd >= 0) close(mc_fd);
            if (rank != 0) {
                const CUresult rc = d.cuMemImportFromShareableHandle(
                    &mc_handle_, reinterpret_cast<void*>(static_cast<uintptr_t>(got)),
                    CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
                close(got);
                check_cu(rc, "cuMemImportFromShareableHandle(multicast)");
            } else {
                close(got);
            }
            check_cu(d.cuMulticastAddDevice(mc_handle_, cu_device(device)), "cuMulticastAddDevice");
            if (barrier) barrier();
            check_cu(d.cuMulticastBindMem(mc_handle_, 0, local_handle_, 0, view_.size, 0), "cuMulticastBindMem");
            mc_bound_ = true;
            void* va = nullptr;
            map_range(mc_handle_, &va);
            view_.mc = static_cast<uint8_t*>(va);
            if (barrier) barrier();
        }
    } catch (...) {
        for (int f : fds) {
            if (f >= 0) close(f);
        }
        release();
        throw;
    }
}

void SymmetricHeap::release() noexcept {
    try {
        const Driver& d = driver();
        cudaSetDevice(device_);
        cudaDeviceSynchronize();
        if (view_.mc) {
            d.cuMemUnmap(reinterpret_cast<CUdeviceptr>(view_.mc), view_.size);
            d.cuMemAddressFree(reinterpret_cast<CUdeviceptr>(view_.mc), view_.size);
            view_.mc = nullptr;
        }
        if (mc_bound_) d.cuMulticastUnbind(mc_handle_, cu_device(device_), 0, view_.size);
        mc_bound_ = false;
        if (mc_handle_) d.cuMemRelease(mc_handle_);
        mc_handle_ = 0;
        bool local_released = false;
        for (int r = 0; r < view_.world; ++r) {
            if (view_.base[r]) {
                d.cuMemUnmap(reinterpret_cast<CUdeviceptr>(view_.base[r]), view_.size);
                d.cuMemAddressFree(reinterpret_cast<CUdeviceptr>(view_.base[r]), view_.size);
                view_.base[r] = nullptr;
            }
            if (r < static_cast<int>(handles_.size()) && handles_[r]) {
                if (handles_[r] == local_handle_) local_released = true;
                d.cuMemRelease(handles_[r]);
                handles_[r] = 0;
            }
        }
        if (local_handle_ && !local_released) d.cuMemRelease(local_handle_);
        local_handle_ = 0;
    } catch (...) {
    }
}

SymmetricHeap::~SymmetricHeap() { release(); }

}  // namespace kiwi::p2p
