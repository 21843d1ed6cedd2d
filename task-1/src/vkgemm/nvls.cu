// NVLink SHARP (NVLS) multicast buffers for the fused all-gather of the row-sharded GEMM.
//
// A multicast object is one virtual range that, through the NVSwitch, stands for the same offset of
// every member GPU's own buffer: a multimem.st to it is replicated by the switch into all members'
// memory.  The GEMM epilogue (vk_gemm_mc) stores every finished box of C once to the multicast
// address of its rows, and the box lands in every GPU's full C at once -- the SMs issue 1/(P-1) of
// the bytes that per-peer stores need.  The reference is single-GPU (README.md:161); this layer is
// new.
//
// Two ways to build a team:
//   * one process, several GPUs (vk_mc_alloc / vk_mc_free): used by vk_gemm_sharded(allgather_c = 4);
//   * one process per GPU (vk_mc_create on one member, vk_mc_import on the others, then
//     vk_mc_attach / vk_mc_detach everywhere): the owner exports the object as a POSIX file
//     descriptor, the others fetch it with pidfd_getfd from the owner's process.
// Memory is created with cuMemCreate (the only memory a multicast object can bind) and mapped twice
// per device: the unicast view (the device's own C) and the multicast view.  Driver entry points
// are resolved through the runtime (cudaGetDriverEntryPoint), so nothing links libcuda directly.
//
// Teardown order matters on a switch fabric: every member must be done with the buffer (the caller
// synchronises and barriers) before any member unmaps and unbinds, and no member may exit while its
// memory is still bound.
#include <cuda.h>
#include <cuda_runtime.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "vkgemm.h"
#include "vk_internal.h"

namespace {

struct DriverApi {
    bool loaded = false;
    CUresult (*DeviceGet)(CUdevice*, int) = nullptr;
    CUresult (*DeviceGetAttribute)(int*, CUdevice_attribute, CUdevice) = nullptr;
    CUresult (*MulticastCreate)(CUmemGenericAllocationHandle*, const CUmulticastObjectProp*) = nullptr;
    CUresult (*MulticastAddDevice)(CUmemGenericAllocationHandle, CUdevice) = nullptr;
    CUresult (*MulticastBindMem)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle, size_t, size_t,
                                 unsigned long long) = nullptr;
    CUresult (*MulticastUnbind)(CUmemGenericAllocationHandle, CUdevice, size_t, size_t) = nullptr;
    CUresult (*MulticastGetGranularity)(size_t*, const CUmulticastObjectProp*, CUmulticastGranularity_flags) = nullptr;
    CUresult (*MemCreate)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long) = nullptr;
    CUresult (*MemRelease)(CUmemGenericAllocationHandle) = nullptr;
    CUresult (*MemGetAllocationGranularity)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags) =
        nullptr;
    CUresult (*MemAddressReserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
    CUresult (*MemAddressFree)(CUdeviceptr, size_t) = nullptr;
    CUresult (*MemMap)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long) = nullptr;
    CUresult (*MemUnmap)(CUdeviceptr, size_t) = nullptr;
    CUresult (*MemSetAccess)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t) = nullptr;
    CUresult (*MemExportToShareableHandle)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType,
                                           unsigned long long) = nullptr;
    CUresult (*MemImportFromShareableHandle)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType) = nullptr;
};
DriverApi g_drv;
std::mutex g_mc_mu;

template <typename F>
bool entry(const char* name, F& fn)
{
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
        p == nullptr)
        return false;
    fn = reinterpret_cast<F>(p);
    return true;
}

int load_driver()
{
    if (g_drv.loaded) return VK_OK;
    DriverApi d;
    const bool ok = entry("cuDeviceGet", d.DeviceGet) && entry("cuDeviceGetAttribute", d.DeviceGetAttribute) &&
                    entry("cuMulticastCreate", d.MulticastCreate) &&
                    entry("cuMulticastAddDevice", d.MulticastAddDevice) &&
                    entry("cuMulticastBindMem", d.MulticastBindMem) && entry("cuMulticastUnbind", d.MulticastUnbind) &&
                    entry("cuMulticastGetGranularity", d.MulticastGetGranularity) &&
                    entry("cuMemCreate", d.MemCreate) && entry("cuMemRelease", d.MemRelease) &&
                    entry("cuMemGetAllocationGranularity", d.MemGetAllocationGranularity) &&
                    entry("cuMemAddressReserve", d.MemAddressReserve) && entry("cuMemAddressFree", d.MemAddressFree) &&
                    entry("cuMemMap", d.MemMap) && entry("cuMemUnmap", d.MemUnmap) &&
                    entry("cuMemSetAccess", d.MemSetAccess) &&
                    entry("cuMemExportToShareableHandle", d.MemExportToShareableHandle) &&
                    entry("cuMemImportFromShareableHandle", d.MemImportFromShareableHandle);
    if (!ok) return vk::set_error(VK_ERR_CUDA, "multicast: a driver entry point is missing (driver too old?)");
    d.loaded = true;
    g_drv = d;
    return VK_OK;
}

int drv_fail(CUresult r, const char* what)
{
    return vk::set_error(VK_ERR_CUDA, "multicast: %s failed (CUresult %d)", what, static_cast<int>(r));
}

#define VK_DRV_TRY(expr, what)                    \
    do {                                          \
        CUresult _r = (expr);                     \
        if (_r != CUDA_SUCCESS) return drv_fail(_r, what); \
    } while (0)

constexpr CUmemAllocationHandleType kShareType = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;

CUmemAllocationProp mem_prop(int dev)
{
    CUmemAllocationProp p;
    memset(&p, 0, sizeof(p));
    p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    p.requestedHandleTypes = kShareType;
    p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    p.location.id = dev;
    return p;
}

// Size rounded up to both the multicast granularity and the device allocation granularity
// (recommended values, both powers of two).
int padded_size(int dev, int members, size_t bytes, size_t* out)
{
    CUmulticastObjectProp mp;
    memset(&mp, 0, sizeof(mp));
    mp.numDevices = static_cast<unsigned>(members);
    mp.size = bytes;
    mp.handleTypes = kShareType;
    size_t g_mc = 0, g_mem = 0;
    VK_DRV_TRY(g_drv.MulticastGetGranularity(&g_mc, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED),
               "cuMulticastGetGranularity");
    const CUmemAllocationProp ap = mem_prop(dev);
    VK_DRV_TRY(g_drv.MemGetAllocationGranularity(&g_mem, &ap, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED),
               "cuMemGetAllocationGranularity");
    size_t g = g_mc > g_mem ? g_mc : g_mem;
    if (g == 0) g = 2u << 20;
    *out = (bytes + g - 1) / g * g;
    return VK_OK;
}

}  // namespace

// One multicast team as seen by this process: the object, and for each local member device its
// physical memory, unicast view and (shared) multicast view.
struct vk_mc_team {
    CUmemGenericAllocationHandle mc = 0;
    int members = 0;
    size_t size = 0;                 // bytes per member (padded)
    int export_fd = -1;              // owner: the exported descriptor; importer: the fetched copy
    std::vector<int> devs;           // local member devices
    std::vector<CUmemGenericAllocationHandle> mem;
    std::vector<CUdeviceptr> uc;     // unicast view per local device
    CUdeviceptr mc_va = 0;           // multicast view (one range, accessible from every local device)
    bool attached = false;
};

namespace {

std::vector<vk_mc_team*> g_teams;  // teams alive in this process (vk_gemm_sharded looks them up)

int set_current(int dev)
{
    const cudaError_t e = cudaSetDevice(dev);
    if (e == cudaSuccess) cudaFree(nullptr);  // make the primary context current for driver calls
    if (e != cudaSuccess) return vk::set_error(VK_ERR_CUDA, "multicast: cudaSetDevice(%d): %s", dev, cudaGetErrorString(e));
    return VK_OK;
}

int check_supported(int dev)
{
    CUdevice cd;
    VK_DRV_TRY(g_drv.DeviceGet(&cd, dev), "cuDeviceGet");
    int mc = 0;
    VK_DRV_TRY(g_drv.DeviceGetAttribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, cd), "cuDeviceGetAttribute");
    if (!mc) return vk::set_error(VK_ERR_UNSUPPORTED, "multicast: device %d does not support NVLS multicast", dev);
    return VK_OK;
}

int create_object(vk_mc_team* t, int dev)
{
    CUmulticastObjectProp mp;
    memset(&mp, 0, sizeof(mp));
    mp.numDevices = static_cast<unsigned>(t->members);
    mp.size = t->size;
    mp.handleTypes = kShareType;
    VK_DRV_TRY(g_drv.MulticastCreate(&t->mc, &mp), "cuMulticastCreate");
    (void)dev;
    return VK_OK;
}

// Adds `dev` to the object, creates and binds its memory and maps its unicast view.  Binding blocks
// until every member device of the team has been added (by this or another process).
int attach_device(vk_mc_team* t, int dev)
{
    int rc = set_current(dev);
    if (rc != VK_OK) return rc;
    CUdevice cd;
    VK_DRV_TRY(g_drv.DeviceGet(&cd, dev), "cuDeviceGet");
    VK_DRV_TRY(g_drv.MulticastAddDevice(t->mc, cd), "cuMulticastAddDevice");
    return VK_OK;
}

int bind_device(vk_mc_team* t, int dev, CUmemGenericAllocationHandle* mem_out, CUdeviceptr* uc_out)
{
    int rc = set_current(dev);
    if (rc != VK_OK) return rc;
    const CUmemAllocationProp ap = mem_prop(dev);
    CUmemGenericAllocationHandle mem = 0;
    VK_DRV_TRY(g_drv.MemCreate(&mem, t->size, &ap, 0), "cuMemCreate");
    CUresult r = g_drv.MulticastBindMem(t->mc, 0, mem, 0, t->size, 0);
    if (r != CUDA_SUCCESS) {
        g_drv.MemRelease(mem);
        return drv_fail(r, "cuMulticastBindMem");
    }
    CUdeviceptr va = 0;
    r = g_drv.MemAddressReserve(&va, t->size, 0, 0, 0);
    if (r == CUDA_SUCCESS) r = g_drv.MemMap(va, t->size, 0, mem, 0);
    if (r == CUDA_SUCCESS) {
        CUmemAccessDesc ad;
        memset(&ad, 0, sizeof(ad));
        ad.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        ad.location.id = dev;
        ad.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
        r = g_drv.MemSetAccess(va, t->size, &ad, 1);
    }
    if (r != CUDA_SUCCESS) {
        CUdevice cd;
        g_drv.DeviceGet(&cd, dev);
        g_drv.MulticastUnbind(t->mc, cd, 0, t->size);
        g_drv.MemRelease(mem);
        return drv_fail(r, "mapping the unicast view");
    }
    *mem_out = mem;
    *uc_out = va;
    return VK_OK;
}

// Maps the multicast view once, readable and writable from every local member device.
int map_multicast(vk_mc_team* t)
{
    VK_DRV_TRY(g_drv.MemAddressReserve(&t->mc_va, t->size, 0, 0, 0), "cuMemAddressReserve (multicast)");
    VK_DRV_TRY(g_drv.MemMap(t->mc_va, t->size, 0, t->mc, 0), "cuMemMap (multicast)");
    std::vector<CUmemAccessDesc> ads(t->devs.size());
    for (size_t i = 0; i < t->devs.size(); ++i) {
        memset(&ads[i], 0, sizeof(ads[i]));
        ads[i].location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        ads[i].location.id = t->devs[i];
        ads[i].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    }
    VK_DRV_TRY(g_drv.MemSetAccess(t->mc_va, t->size, ads.data(), ads.size()), "cuMemSetAccess (multicast)");
    return VK_OK;
}

// Unmaps both views, unbinds and releases this process's share of the team (best effort: every
// step runs even when an earlier one failed; the first failure is reported).
int teardown(vk_mc_team* t)
{
    int rc = VK_OK;
    auto note = [&](CUresult r, const char* what) {
        if (r != CUDA_SUCCESS && rc == VK_OK) rc = drv_fail(r, what);
    };
    for (int d : t->devs) {
        if (set_current(d) == VK_OK) cudaDeviceSynchronize();
    }
    if (t->mc_va != 0) {
        note(g_drv.MemUnmap(t->mc_va, t->size), "cuMemUnmap (multicast)");
        note(g_drv.MemAddressFree(t->mc_va, t->size), "cuMemAddressFree (multicast)");
        t->mc_va = 0;
    }
    for (size_t i = 0; i < t->devs.size(); ++i) {
        if (i < t->uc.size() && t->uc[i] != 0) {
            note(g_drv.MemUnmap(t->uc[i], t->size), "cuMemUnmap");
            note(g_drv.MemAddressFree(t->uc[i], t->size), "cuMemAddressFree");
        }
        if (i < t->mem.size() && t->mem[i] != 0) {
            CUdevice cd;
            if (g_drv.DeviceGet(&cd, t->devs[i]) == CUDA_SUCCESS)
                note(g_drv.MulticastUnbind(t->mc, cd, 0, t->size), "cuMulticastUnbind");
            note(g_drv.MemRelease(t->mem[i]), "cuMemRelease");
        }
    }
    t->uc.clear();
    t->mem.clear();
    if (t->mc != 0) {
        note(g_drv.MemRelease(t->mc), "cuMemRelease (multicast object)");
        t->mc = 0;
    }
    if (t->export_fd >= 0) {
        close(t->export_fd);
        t->export_fd = -1;
    }
    t->attached = false;
    return rc;
}

void forget(vk_mc_team* t)
{
    for (size_t i = 0; i < g_teams.size(); ++i)
        if (g_teams[i] == t) {
            g_teams.erase(g_teams.begin() + static_cast<long>(i));
            break;
        }
}

}  // namespace

namespace vk {
// Multicast address of `ptr` on device `dev` if it lies in the unicast view of a live team, else
// nullptr (vk_gemm_sharded's NVLS mode).
void* mc_lookup(int dev, const void* ptr, size_t bytes)
{
    std::lock_guard<std::mutex> lk(g_mc_mu);
    const CUdeviceptr p = reinterpret_cast<CUdeviceptr>(ptr);
    for (vk_mc_team* t : g_teams) {
        if (!t->attached) continue;
        for (size_t i = 0; i < t->devs.size(); ++i) {
            if (t->devs[i] != dev || i >= t->uc.size()) continue;
            if (p >= t->uc[i] && p + bytes <= t->uc[i] + t->size)
                return reinterpret_cast<void*>(t->mc_va + (p - t->uc[i]));
        }
    }
    return nullptr;
}
}  // namespace vk

extern "C" int vk_mc_supported(int device, int* out)
{
    if (out == nullptr) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_mc_supported: out is NULL");
    *out = 0;
    std::lock_guard<std::mutex> lk(g_mc_mu);
    int rc = load_driver();
    if (rc != VK_OK) return rc;
    int prev = 0;
    cudaGetDevice(&prev);
    rc = set_current(device);
    if (rc == VK_OK) {
        CUdevice cd;
        int v = 0;
        if (g_drv.DeviceGet(&cd, device) == CUDA_SUCCESS &&
            g_drv.DeviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, cd) == CUDA_SUCCESS)
            *out = v ? 1 : 0;
    }
    cudaSetDevice(prev);
    return rc;
}

extern "C" int vk_mc_alloc(int32_t ndev, const int32_t* devices, size_t bytes, void** ptrs, void** mc_ptr)
{
    if (ndev < 1 || ndev > 64 || devices == nullptr || ptrs == nullptr || mc_ptr == nullptr || bytes == 0)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_mc_alloc: bad arguments");
    std::lock_guard<std::mutex> lk(g_mc_mu);
    int rc = load_driver();
    if (rc != VK_OK) return rc;
    int prev = 0;
    cudaGetDevice(&prev);
    vk_mc_team* t = new vk_mc_team();
    t->members = ndev;
    t->devs.assign(devices, devices + ndev);
    for (int i = 0; i < ndev && rc == VK_OK; ++i) rc = check_supported(devices[i]);
    if (rc == VK_OK) rc = set_current(devices[0]);
    if (rc == VK_OK) rc = padded_size(devices[0], ndev, bytes, &t->size);
    if (rc == VK_OK) rc = create_object(t, devices[0]);
    for (int i = 0; i < ndev && rc == VK_OK; ++i) rc = attach_device(t, devices[i]);
    for (int i = 0; i < ndev && rc == VK_OK; ++i) {
        CUmemGenericAllocationHandle mem = 0;
        CUdeviceptr uc = 0;
        rc = bind_device(t, devices[i], &mem, &uc);
        if (rc == VK_OK) {
            t->mem.push_back(mem);
            t->uc.push_back(uc);
        }
    }
    if (rc == VK_OK) rc = set_current(devices[0]);
    if (rc == VK_OK) rc = map_multicast(t);
    if (rc != VK_OK) {
        teardown(t);
        delete t;
        cudaSetDevice(prev);
        return rc;
    }
    t->attached = true;
    g_teams.push_back(t);
    for (int i = 0; i < ndev; ++i) ptrs[i] = reinterpret_cast<void*>(t->uc[i]);
    *mc_ptr = reinterpret_cast<void*>(t->mc_va);
    cudaSetDevice(prev);
    return VK_OK;
}

extern "C" int vk_mc_free(void* mc_ptr)
{
    std::lock_guard<std::mutex> lk(g_mc_mu);
    for (vk_mc_team* t : g_teams) {
        if (reinterpret_cast<void*>(t->mc_va) != mc_ptr) continue;
        int prev = 0;
        cudaGetDevice(&prev);
        const int rc = teardown(t);
        forget(t);
        delete t;
        cudaSetDevice(prev);
        return rc;
    }
    return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_mc_free: not a multicast pointer from vk_mc_alloc");
}

extern "C" int vk_mc_create(int device, int32_t members, size_t bytes, vk_mc_team** team, int64_t* share)
{
    if (team == nullptr || share == nullptr || members < 1 || members > 64 || bytes == 0)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_mc_create: bad arguments");
    std::lock_guard<std::mutex> lk(g_mc_mu);
    int rc = load_driver();
    if (rc != VK_OK) return rc;
    rc = set_current(device);
    if (rc == VK_OK) rc = check_supported(device);
    vk_mc_team* t = new vk_mc_team();
    t->members = members;
    t->devs.push_back(device);
    if (rc == VK_OK) rc = padded_size(device, members, bytes, &t->size);
    if (rc == VK_OK) rc = create_object(t, device);
    if (rc == VK_OK) {
        int fd = -1;
        const CUresult r = g_drv.MemExportToShareableHandle(&fd, t->mc, kShareType, 0);
        if (r != CUDA_SUCCESS) rc = drv_fail(r, "cuMemExportToShareableHandle");
        t->export_fd = fd;
    }
    if (rc != VK_OK) {
        teardown(t);
        delete t;
        return rc;
    }
    g_teams.push_back(t);
    share[0] = static_cast<int64_t>(getpid());
    share[1] = static_cast<int64_t>(t->export_fd);
    share[2] = static_cast<int64_t>(t->size);
    *team = t;
    return VK_OK;
}

extern "C" int vk_mc_import(int device, int32_t members, const int64_t* share, vk_mc_team** team)
{
    if (team == nullptr || share == nullptr || members < 1 || members > 64)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_mc_import: bad arguments");
    std::lock_guard<std::mutex> lk(g_mc_mu);
    int rc = load_driver();
    if (rc != VK_OK) return rc;
    rc = set_current(device);
    if (rc == VK_OK) rc = check_supported(device);
    if (rc != VK_OK) return rc;
    // The owner's descriptor is fetched out of its process (same node, same user).
    const long pidfd = syscall(SYS_pidfd_open, static_cast<pid_t>(share[0]), 0);
    if (pidfd < 0) return vk::set_error(VK_ERR_CUDA, "vk_mc_import: pidfd_open(%lld) failed", (long long)share[0]);
    const long fd = syscall(SYS_pidfd_getfd, static_cast<int>(pidfd), static_cast<int>(share[1]), 0);
    close(static_cast<int>(pidfd));
    if (fd < 0) return vk::set_error(VK_ERR_CUDA, "vk_mc_import: pidfd_getfd(%lld) failed", (long long)share[1]);
    vk_mc_team* t = new vk_mc_team();
    t->members = members;
    t->size = static_cast<size_t>(share[2]);
    t->export_fd = static_cast<int>(fd);
    t->devs.push_back(device);
    const CUresult r = g_drv.MemImportFromShareableHandle(&t->mc, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                                                          kShareType);
    if (r != CUDA_SUCCESS) {
        rc = drv_fail(r, "cuMemImportFromShareableHandle");
        teardown(t);
        delete t;
        return rc;
    }
    g_teams.push_back(t);
    *team = t;
    return VK_OK;
}

extern "C" int vk_mc_attach(vk_mc_team* t, void** local_ptr, void** mc_ptr, size_t* size)
{
    if (t == nullptr || local_ptr == nullptr || mc_ptr == nullptr)
        return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_mc_attach: NULL");
    std::lock_guard<std::mutex> lk(g_mc_mu);
    if (t->attached) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_mc_attach: already attached");
    const int dev = t->devs[0];
    int rc = attach_device(t, dev);
    CUmemGenericAllocationHandle mem = 0;
    CUdeviceptr uc = 0;
    if (rc == VK_OK) rc = bind_device(t, dev, &mem, &uc);
    if (rc == VK_OK) {
        t->mem.push_back(mem);
        t->uc.push_back(uc);
        rc = map_multicast(t);
        if (rc != VK_OK) {
            // undo this member's mapping and binding at once, so that it never leaves with memory bound;
            // the object itself is released by vk_mc_detach
            if (t->mc_va != 0) {
                g_drv.MemUnmap(t->mc_va, t->size);
                g_drv.MemAddressFree(t->mc_va, t->size);
                t->mc_va = 0;
            }
            g_drv.MemUnmap(uc, t->size);
            g_drv.MemAddressFree(uc, t->size);
            CUdevice cd;
            if (g_drv.DeviceGet(&cd, dev) == CUDA_SUCCESS) g_drv.MulticastUnbind(t->mc, cd, 0, t->size);
            g_drv.MemRelease(mem);
            t->mem.clear();
            t->uc.clear();
        }
    }
    if (rc != VK_OK) return rc;
    t->attached = true;
    *local_ptr = reinterpret_cast<void*>(t->uc[0]);
    *mc_ptr = reinterpret_cast<void*>(t->mc_va);
    if (size) *size = t->size;
    return VK_OK;
}

extern "C" int vk_mc_detach(vk_mc_team* t)
{
    if (t == nullptr) return vk::set_error(VK_ERR_INVALID_ARGUMENT, "vk_mc_detach: NULL");
    std::lock_guard<std::mutex> lk(g_mc_mu);
    int prev = 0;
    cudaGetDevice(&prev);
    const int rc = teardown(t);
    forget(t);
    delete t;
    cudaSetDevice(prev);
    return rc;
}
