// Host side of NVLS multicast memory (see nvls.h for the protocol).
#include "nvls.h"

#include <cuda_runtime.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstddef>
#include <cstring>
#include <stdexcept>
#include <thread>

namespace mnb {
namespace {

// ---- driver entry points -------------------------------------------------------

struct Driver {
  decltype(&cuGetErrorString) get_error_string = nullptr;
  decltype(&cuDeviceGet) device_get = nullptr;
  decltype(&cuDeviceGetAttribute) device_get_attribute = nullptr;
  decltype(&cuMulticastGetGranularity) mc_granularity = nullptr;
  decltype(&cuMulticastCreate) mc_create = nullptr;
  decltype(&cuMulticastAddDevice) mc_add_device = nullptr;
  decltype(&cuMulticastBindMem) mc_bind_mem = nullptr;
  decltype(&cuMulticastUnbind) mc_unbind = nullptr;
  decltype(&cuMemGetAllocationGranularity) mem_granularity = nullptr;
  decltype(&cuMemCreate) mem_create = nullptr;
  decltype(&cuMemRelease) mem_release = nullptr;
  decltype(&cuMemAddressReserve) addr_reserve = nullptr;
  decltype(&cuMemAddressFree) addr_free = nullptr;
  decltype(&cuMemMap) mem_map = nullptr;
  decltype(&cuMemUnmap) mem_unmap = nullptr;
  decltype(&cuMemSetAccess) mem_set_access = nullptr;
  decltype(&cuMemExportToShareableHandle) mem_export = nullptr;
  decltype(&cuMemImportFromShareableHandle) mem_import = nullptr;
  std::string missing;
};

template <typename F>
void resolve(F* slot, const char* name, std::string* missing) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
      p == nullptr) {
    if (!missing->empty()) *missing += ", ";
    *missing += name;
    p = nullptr;
  }
  *slot = reinterpret_cast<F>(p);
}

const Driver& drv() {
  static const Driver d = [] {
    Driver x;
    resolve(&x.get_error_string, "cuGetErrorString", &x.missing);
    resolve(&x.device_get, "cuDeviceGet", &x.missing);
    resolve(&x.device_get_attribute, "cuDeviceGetAttribute", &x.missing);
    resolve(&x.mc_granularity, "cuMulticastGetGranularity", &x.missing);
    resolve(&x.mc_create, "cuMulticastCreate", &x.missing);
    resolve(&x.mc_add_device, "cuMulticastAddDevice", &x.missing);
    resolve(&x.mc_bind_mem, "cuMulticastBindMem", &x.missing);
    resolve(&x.mc_unbind, "cuMulticastUnbind", &x.missing);
    resolve(&x.mem_granularity, "cuMemGetAllocationGranularity", &x.missing);
    resolve(&x.mem_create, "cuMemCreate", &x.missing);
    resolve(&x.mem_release, "cuMemRelease", &x.missing);
    resolve(&x.addr_reserve, "cuMemAddressReserve", &x.missing);
    resolve(&x.addr_free, "cuMemAddressFree", &x.missing);
    resolve(&x.mem_map, "cuMemMap", &x.missing);
    resolve(&x.mem_unmap, "cuMemUnmap", &x.missing);
    resolve(&x.mem_set_access, "cuMemSetAccess", &x.missing);
    resolve(&x.mem_export, "cuMemExportToShareableHandle", &x.missing);
    resolve(&x.mem_import, "cuMemImportFromShareableHandle", &x.missing);
    return x;
  }();
  return d;
}

void cu_check(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return;
  const char* msg = nullptr;
  if (drv().get_error_string != nullptr) drv().get_error_string(r, &msg);
  throw std::runtime_error(std::string("NVLS: ") + what + " failed: " + (msg ? msg : "unknown error") + " (" +
                           std::to_string(static_cast<int>(r)) + ")");
}

CUdevice cu_device(int ordinal) {
  CUdevice dev = 0;
  cu_check(drv().device_get(&dev, ordinal), "cuDeviceGet");
  return dev;
}

// ---- file descriptors over abstract Unix sockets --------------------------------

std::atomic<int> g_sock_counter{0};

sockaddr_un abstract_addr(const std::string& name, socklen_t* len) {
  sockaddr_un addr{};
  addr.sun_family = AF_UNIX;
  if (name.size() + 1 > sizeof(addr.sun_path)) throw std::runtime_error("NVLS: socket name too long");
  addr.sun_path[0] = '\0';  // abstract namespace: nothing on the file system
  std::memcpy(addr.sun_path + 1, name.data(), name.size());
  *len = static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + name.size());
  return addr;
}

void send_fd(const std::string& name, int fd, double timeout_s) {
  socklen_t len = 0;
  const sockaddr_un addr = abstract_addr(name, &len);
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
  int s = -1;
  for (;;) {
    s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (s < 0) throw std::runtime_error(std::string("NVLS: socket(): ") + std::strerror(errno));
    if (connect(s, reinterpret_cast<const sockaddr*>(&addr), len) == 0) break;
    const int err = errno;
    close(s);
    if (std::chrono::steady_clock::now() > deadline)
      throw std::runtime_error(std::string("NVLS: could not reach a peer's socket: ") + std::strerror(err));
    std::this_thread::sleep_for(std::chrono::milliseconds(5));
  }
  char byte = 'm';
  iovec iov{&byte, 1};
  alignas(cmsghdr) char control[CMSG_SPACE(sizeof(int))] = {};
  msghdr msg{};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = control;
  msg.msg_controllen = sizeof(control);
  cmsghdr* c = CMSG_FIRSTHDR(&msg);
  c->cmsg_level = SOL_SOCKET;
  c->cmsg_type = SCM_RIGHTS;
  c->cmsg_len = CMSG_LEN(sizeof(int));
  std::memcpy(CMSG_DATA(c), &fd, sizeof(int));
  const ssize_t sent = sendmsg(s, &msg, 0);
  const int err = errno;
  close(s);
  if (sent != 1) throw std::runtime_error(std::string("NVLS: sendmsg(): ") + std::strerror(err));
}

int recv_fd(int listen_fd, double timeout_s) {
  pollfd p{listen_fd, POLLIN, 0};
  const int ready = poll(&p, 1, static_cast<int>(timeout_s * 1000));
  if (ready <= 0) throw std::runtime_error("NVLS: timed out waiting for rank 0's multicast handle");
  const int s = accept4(listen_fd, nullptr, nullptr, SOCK_CLOEXEC);
  if (s < 0) throw std::runtime_error(std::string("NVLS: accept(): ") + std::strerror(errno));
  char byte = 0;
  iovec iov{&byte, 1};
  alignas(cmsghdr) char control[CMSG_SPACE(sizeof(int))] = {};
  msghdr msg{};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = control;
  msg.msg_controllen = sizeof(control);
  const ssize_t got = recvmsg(s, &msg, 0);
  const int err = errno;
  close(s);
  if (got != 1) throw std::runtime_error(std::string("NVLS: recvmsg(): ") + std::strerror(err));
  cmsghdr* c = CMSG_FIRSTHDR(&msg);
  if (c == nullptr || c->cmsg_type != SCM_RIGHTS) throw std::runtime_error("NVLS: no descriptor in the message");
  int fd = -1;
  std::memcpy(&fd, CMSG_DATA(c), sizeof(int));
  return fd;
}

int64_t round_up(int64_t x, int64_t q) { return (x + q - 1) / q * q; }

}  // namespace

std::string nvls_unsupported_reason(int device) {
  const Driver& d = drv();
  if (!d.missing.empty()) return "driver lacks " + d.missing;
  CUdevice dev = 0;
  if (d.device_get(&dev, device) != CUDA_SUCCESS) return "cuDeviceGet failed";
  int mc = 0;
  if (d.device_get_attribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev) != CUDA_SUCCESS)
    return "cannot query CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED";
  if (!mc) return "the device does not support multicast objects";
  return "";
}

NvlsObject::NvlsObject(int rank, int world, int device, int64_t bytes) : rank_(rank), world_(world), device_(device) {
  try {
    create(bytes);
  } catch (...) {
    release();  // a constructor that throws runs no destructor
    throw;
  }
}

void NvlsObject::create(int64_t bytes) {
  const Driver& d = drv();
  if (!d.missing.empty()) throw std::runtime_error("NVLS: driver lacks " + d.missing);
  const CUdevice dev = cu_device(device_);
  CUmulticastObjectProp mp{};
  mp.numDevices = static_cast<unsigned>(world_);
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  mp.size = static_cast<size_t>(bytes);
  size_t mc_gran = 0;
  cu_check(d.mc_granularity(&mc_gran, &mp, CU_MULTICAST_GRANULARITY_MINIMUM), "cuMulticastGetGranularity");
  CUmemAllocationProp ap{};
  ap.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  ap.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  ap.location.id = dev;
  ap.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  size_t mem_gran = 0;
  cu_check(d.mem_granularity(&mem_gran, &ap, CU_MEM_ALLOC_GRANULARITY_MINIMUM), "cuMemGetAllocationGranularity");
  const int64_t gran = static_cast<int64_t>(std::max(mc_gran, mem_gran));
  gran_ = gran;
  bytes_ = round_up(std::max<int64_t>(bytes, 1), gran);
  mp.size = static_cast<size_t>(bytes_);
  if (rank_ == 0) {
    cu_check(d.mc_create(&mc_handle_, &mp), "cuMulticastCreate");
    have_mc_ = true;
    cu_check(d.mem_export(&export_fd_, mc_handle_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
             "cuMemExportToShareableHandle(multicast)");
  }
  cu_check(d.mem_create(&mem_handle_, static_cast<size_t>(bytes_), &ap, 0), "cuMemCreate");
  have_mem_ = true;
  listen_fd_ = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (listen_fd_ < 0) throw std::runtime_error(std::string("NVLS: socket(): ") + std::strerror(errno));
  sock_name_ = "mnb-nvls-" + std::to_string(getpid()) + "-" + std::to_string(g_sock_counter.fetch_add(1)) + "-r" +
               std::to_string(rank_);
  socklen_t len = 0;
  const sockaddr_un addr = abstract_addr(sock_name_, &len);
  if (bind(listen_fd_, reinterpret_cast<const sockaddr*>(&addr), len) != 0 || listen(listen_fd_, world_) != 0)
    throw std::runtime_error(std::string("NVLS: cannot listen on a Unix socket: ") + std::strerror(errno));
}

void NvlsObject::exchange(const std::vector<std::string>& names, double timeout_s) {
  const Driver& d = drv();
  if (static_cast<int>(names.size()) != world_) throw std::runtime_error("NVLS: need one socket name per rank");
  if (rank_ == 0) {
    for (int r = 1; r < world_; ++r) send_fd(names[r], export_fd_, timeout_s);
  } else {
    const int fd = recv_fd(listen_fd_, timeout_s);
    const CUresult res =
        d.mem_import(&mc_handle_, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                     CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
    close(fd);
    cu_check(res, "cuMemImportFromShareableHandle(multicast)");
    have_mc_ = true;
  }
  cu_check(d.mc_add_device(mc_handle_, cu_device(device_)), "cuMulticastAddDevice");
  added_ = true;
}

void NvlsObject::bind_and_map() {
  const Driver& d = drv();
  const CUdevice dev = cu_device(device_);
  cu_check(d.mc_bind_mem(mc_handle_, 0, mem_handle_, 0, static_cast<size_t>(bytes_), 0), "cuMulticastBindMem");
  bound_ = true;
  CUmemAccessDesc access{};
  access.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  access.location.id = dev;
  access.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  CUdeviceptr uc = 0, mc = 0;
  cu_check(d.addr_reserve(&uc, static_cast<size_t>(bytes_), static_cast<size_t>(gran_), 0, 0),
           "cuMemAddressReserve(unicast)");
  uc_ = reinterpret_cast<void*>(uc);
  cu_check(d.mem_map(uc, static_cast<size_t>(bytes_), 0, mem_handle_, 0), "cuMemMap(unicast)");
  uc_mapped_ = true;
  cu_check(d.mem_set_access(uc, static_cast<size_t>(bytes_), &access, 1), "cuMemSetAccess(unicast)");
  cu_check(d.addr_reserve(&mc, static_cast<size_t>(bytes_), static_cast<size_t>(gran_), 0, 0),
           "cuMemAddressReserve(multicast)");
  mc_ = reinterpret_cast<void*>(mc);
  cu_check(d.mem_map(mc, static_cast<size_t>(bytes_), 0, mc_handle_, 0), "cuMemMap(multicast)");
  mc_mapped_ = true;
  cu_check(d.mem_set_access(mc, static_cast<size_t>(bytes_), &access, 1), "cuMemSetAccess(multicast)");
  mapped_ = true;
  if (cudaMemset(uc_, 0, static_cast<size_t>(bytes_)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
    throw std::runtime_error("NVLS: cannot clear the bound memory");
}

void NvlsObject::release() {
  const Driver& d = drv();
  if (d.mem_unmap == nullptr) return;
  const size_t n = static_cast<size_t>(bytes_);
  // each address is unmapped on its own flag: a set-up that failed between the
  // two mappings leaves one of them mapped
  if (mc_ != nullptr) {
    if (mc_mapped_) d.mem_unmap(reinterpret_cast<CUdeviceptr>(mc_), n);
    d.addr_free(reinterpret_cast<CUdeviceptr>(mc_), n);
    mc_ = nullptr;
  }
  if (uc_ != nullptr) {
    if (uc_mapped_) d.mem_unmap(reinterpret_cast<CUdeviceptr>(uc_), n);
    d.addr_free(reinterpret_cast<CUdeviceptr>(uc_), n);
    uc_ = nullptr;
  }
  uc_mapped_ = mc_mapped_ = mapped_ = false;
  if (bound_) {
    CUdevice dev = 0;
    if (d.device_get(&dev, device_) == CUDA_SUCCESS) d.mc_unbind(mc_handle_, dev, 0, n);
    bound_ = false;
  }
  if (have_mem_) {
    d.mem_release(mem_handle_);
    have_mem_ = false;
  }
  if (have_mc_) {
    d.mem_release(mc_handle_);
    have_mc_ = false;
  }
  if (export_fd_ >= 0) close(export_fd_);
  export_fd_ = -1;
  if (listen_fd_ >= 0) close(listen_fd_);
  listen_fd_ = -1;
}

NvlsObject::~NvlsObject() {
  try {
    release();
  } catch (...) {
  }
}

}  // namespace mnb
