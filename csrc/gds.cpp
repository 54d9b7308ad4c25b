// GPUDirect Storage reads through NVIDIA cuFile (reference src/strix/cufile_ffi.rs,
// src/strix/gpu_direct.rs:540-640): file ranges read straight into device memory.
//
// libcufile is opened with dlopen on first use, so the extension imports (and the
// threaded-pread fallback keeps working) where the library or the nvidia-fs driver is
// missing. Without nvidia-fs, cuFile runs in its compatibility mode (POSIX reads through
// its own pinned bounce buffers); with it, the NVMe DMA lands in HBM directly.
// One reader holds one registered file; device buffers may be registered for the fastest
// path (cuFileBufRegister) or passed unregistered.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <cufile.h>
#include <dlfcn.h>
#include <fcntl.h>
#include <unistd.h>

#include <cstdlib>
#include <mutex>
#include <string>

namespace {

struct CuFileApi {
  CUfileError_t (*driver_open)() = nullptr;
  CUfileError_t (*handle_register)(CUfileHandle_t*, CUfileDescr_t*) = nullptr;
  void (*handle_deregister)(CUfileHandle_t) = nullptr;
  CUfileError_t (*buf_register)(const void*, size_t, int) = nullptr;
  CUfileError_t (*buf_deregister)(const void*) = nullptr;
  ssize_t (*read)(CUfileHandle_t, void*, size_t, off_t, off_t) = nullptr;
  std::string error;
  bool ok = false;
};

CuFileApi& api() {
  static CuFileApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    // Off unless AIR_CUFILE=1: on the B200 pool used for testing (no nvidia-fs driver) a
    // cuFile read in compatibility mode did not return, so nothing here runs by default.
    const char* en = getenv("AIR_CUFILE");
    if (!(en && en[0] == '1')) {
      a.error = "cuFile disabled (set AIR_CUFILE=1 to enable)";
      return;
    }
    void* h = dlopen("libcufile.so.0", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libcufile.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      a.error = std::string("libcufile not found: ") + dlerror();
      return;
    }
    auto sym = [&](const char* n) { return dlsym(h, n); };
    a.driver_open = reinterpret_cast<decltype(a.driver_open)>(sym("cuFileDriverOpen"));
    a.handle_register = reinterpret_cast<decltype(a.handle_register)>(sym("cuFileHandleRegister"));
    a.handle_deregister = reinterpret_cast<decltype(a.handle_deregister)>(sym("cuFileHandleDeregister"));
    a.buf_register = reinterpret_cast<decltype(a.buf_register)>(sym("cuFileBufRegister"));
    a.buf_deregister = reinterpret_cast<decltype(a.buf_deregister)>(sym("cuFileBufDeregister"));
    a.read = reinterpret_cast<decltype(a.read)>(sym("cuFileRead"));
    if (!a.driver_open || !a.handle_register || !a.handle_deregister || !a.read || !a.buf_register ||
        !a.buf_deregister) {
      a.error = "libcufile lacks an expected symbol";
      return;
    }
    const CUfileError_t e = a.driver_open();
    if (e.err != CU_FILE_SUCCESS) {
      a.error = std::string("cuFileDriverOpen: ") + CUFILE_ERRSTR(e.err);
      return;
    }
    a.ok = true;
  });
  return a;
}

class GdsReader {
 public:
  explicit GdsReader(const std::string& path) {
    CuFileApi& a = api();
    TORCH_CHECK(a.ok, "cuFile unavailable: ", a.error);
    fd_ = open(path.c_str(), O_RDONLY | O_DIRECT);
    if (fd_ < 0) fd_ = open(path.c_str(), O_RDONLY);   // file systems without O_DIRECT: compat mode
    TORCH_CHECK(fd_ >= 0, "GdsReader: cannot open ", path);
    CUfileDescr_t d{};
    d.handle.fd = fd_;
    d.type = CU_FILE_HANDLE_TYPE_OPAQUE_FD;
    const CUfileError_t e = a.handle_register(&fh_, &d);
    if (e.err != CU_FILE_SUCCESS) {
      close(fd_);
      fd_ = -1;
      TORCH_CHECK(false, "cuFileHandleRegister: ", CUFILE_ERRSTR(e.err));
    }
  }
  ~GdsReader() { close_file(); }

  void close_file() {
    if (fd_ >= 0) {
      api().handle_deregister(fh_);
      close(fd_);
      fd_ = -1;
    }
  }

  // Read `nbytes` at `file_offset` into dst (a CUDA tensor) at byte `dst_offset`. Returns
  // the bytes read (short only at end of file).
  int64_t read(at::Tensor dst, int64_t file_offset, int64_t nbytes, int64_t dst_offset) {
    TORCH_CHECK(fd_ >= 0, "GdsReader: closed");
    TORCH_CHECK(dst.is_cuda() && dst.is_contiguous(), "GdsReader.read: contiguous CUDA destination");
    TORCH_CHECK(dst_offset >= 0 && nbytes >= 0 && dst_offset + nbytes <= (int64_t)dst.nbytes(),
                "GdsReader.read: destination range out of bounds");
    c10::cuda::CUDAGuard g(dst.device());
    int64_t done = 0;
    while (done < nbytes) {
      const ssize_t r = api().read(fh_, dst.data_ptr(), (size_t)(nbytes - done), (off_t)(file_offset + done),
                                   (off_t)(dst_offset + done));
      TORCH_CHECK(r >= 0, "cuFileRead failed (", r, ")");
      if (r == 0) break;
      done += r;
    }
    return done;
  }

 private:
  int fd_ = -1;
  CUfileHandle_t fh_ = nullptr;
};

}  // namespace

void register_gds(pybind11::module_& m) {
  m.def("gds_available", [] { return api().ok; });
  m.def("gds_error", [] { return api().error; });
  m.def("gds_buf_register", [](at::Tensor t) {
    TORCH_CHECK(api().ok, "cuFile unavailable: ", api().error);
    const CUfileError_t e = api().buf_register(t.data_ptr(), t.nbytes(), 0);
    return e.err == CU_FILE_SUCCESS;
  });
  m.def("gds_buf_deregister", [](at::Tensor t) {
    if (api().ok) api().buf_deregister(t.data_ptr());
  });
  pybind11::class_<GdsReader>(m, "GdsReader")
      .def(pybind11::init<const std::string&>())
      .def("read", &GdsReader::read)
      .def("close", &GdsReader::close_file);
}
