// NVLink SHARP (NVLS) multicast memory for the device communicator.
//
// One NvlsObject is a multicast object that spans every rank of a device
// communicator, with `bytes` of this GPU's memory bound to it and mapped
// twice in this process:
//   uc()  the ordinary (unicast) address of the local memory;
//   mc()  the multicast address.  A `multimem.st` to mc()+off writes every
//         rank's memory at off; a `multimem.ld_reduce` from mc()+off returns
//         the sum (min, max) over every rank's value at off, reduced inside
//         the NVSwitch.
// Building one is collective and takes three steps with host barriers in
// between (the Python layer drives them over the host communicator):
//   1. constructor: rank 0 creates the multicast object and exports it as a
//      POSIX file descriptor; every rank opens a listening Unix socket;
//   2. exchange(): rank 0 sends the descriptor to every other rank over its
//      socket (SCM_RIGHTS); each rank imports it and adds its own device;
//   3. bind_and_map(): once every device is in, each rank binds its memory and
//      maps both addresses.
// release() undoes it; the caller synchronises every rank first, because a
// rank that unbinds while a peer's kernel still reads the object through the
// switch faults that peer.
//
// Driver entry points are resolved at run time through
// cudaGetDriverEntryPoint, so the library does not link libcuda and still
// loads on a machine without a GPU driver.
#pragma once

#include <cuda.h>

#include <cstdint>
#include <string>
#include <vector>

namespace mnb {

// Why NVLS is unusable on `device` ("" when it is usable).
std::string nvls_unsupported_reason(int device);

class NvlsObject {
 public:
  NvlsObject(int rank, int world, int device, int64_t bytes);
  ~NvlsObject();
  NvlsObject(const NvlsObject&) = delete;
  NvlsObject& operator=(const NvlsObject&) = delete;

  const std::string& socket_name() const { return sock_name_; }
  void exchange(const std::vector<std::string>& names, double timeout_s);
  void bind_and_map();
  void release();

  void* uc() const { return uc_; }
  void* mc() const { return mc_; }
  int64_t bytes() const { return bytes_; }
  bool mapped() const { return mapped_; }

 private:
  void create(int64_t bytes);

  int rank_, world_, device_;
  int64_t bytes_ = 0;
  int64_t gran_ = 0;  // mapping granularity (multicast and allocation)
  CUmemGenericAllocationHandle mc_handle_ = 0;
  CUmemGenericAllocationHandle mem_handle_ = 0;
  bool have_mc_ = false, have_mem_ = false, added_ = false, bound_ = false, mapped_ = false;
  bool uc_mapped_ = false, mc_mapped_ = false;
  int export_fd_ = -1;
  int listen_fd_ = -1;
  std::string sock_name_;
  void* uc_ = nullptr;
  void* mc_ = nullptr;
};

}  // namespace mnb
