// CUDA driver entry points used by the symmetric heap (VMM + multicast),
// resolved at run time through cudaGetDriverEntryPoint so the extension never
// links libcuda directly and still imports on a machine without a GPU driver.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

namespace kiwi::p2p {

struct Driver {
    PFN_cuMemCreate_v10020 cuMemCreate = nullptr;
    PFN_cuMemRelease_v10020 cuMemRelease = nullptr;
    PFN_cuMemExportToShareableHandle_v10020 cuMemExportToShareableHandle = nullptr;
    PFN_cuMemImportFromShareableHandle_v10020 cuMemImportFromShareableHandle = nullptr;
    PFN_cuMemAddressReserve_v10020 cuMemAddressReserve = nullptr;
    PFN_cuMemAddressFree_v10020 cuMemAddressFree = nullptr;
    PFN_cuMemMap_v10020 cuMemMap = nullptr;
    PFN_cuMemUnmap_v10020 cuMemUnmap = nullptr;
    PFN_cuMemSetAccess_v10020 cuMemSetAccess = nullptr;
    PFN_cuMemGetAllocationGranularity_v10020 cuMemGetAllocationGranularity = nullptr;
    PFN_cuMulticastCreate_v12010 cuMulticastCreate = nullptr;
    PFN_cuMulticastAddDevice_v12010 cuMulticastAddDevice = nullptr;
    PFN_cuMulticastBindMem_v12010 cuMulticastBindMem = nullptr;
    PFN_cuMulticastUnbind_v12010 cuMulticastUnbind = nullptr;
    PFN_cuMulticastGetGranularity_v12010 cuMulticastGetGranularity = nullptr;
    PFN_cuDeviceGetAttribute_v2000 cuDeviceGetAttribute = nullptr;
    PFN_cuDeviceGet_v2000 cuDeviceGet = nullptr;
    PFN_cuGetErrorString_v6000 cuGetErrorString = nullptr;
    PFN_cuCtxGetCurrent_v4000 cuCtxGetCurrent = nullptr;
    PFN_cuStreamWriteValue64_v11070 cuStreamWriteValue64 = nullptr;
    PFN_cuStreamWaitValue64_v11070 cuStreamWaitValue64 = nullptr;
};

/// Loads the entry points once (throws kiwi::error if the driver lacks one).
const Driver& driver();

/// Throws kiwi::error with the driver's message when `r` is not CUDA_SUCCESS.
void check_cu(CUresult r, const char* what);

}  // namespace kiwi::p2p
