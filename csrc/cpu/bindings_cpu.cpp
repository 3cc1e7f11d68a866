// Python bindings of the host-only native runtime (no CUDA needed):
// the CPU mailbox allreduce engine and the FD-exchange helpers.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "fdx.h"
#include "mailbox_cpu.h"

namespace py = pybind11;

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "host runtime: CPU mailbox allreduce engine + FD exchange";
  py::class_<mbx::CpuMailbox>(m, "CpuMailbox")
      .def(py::init<const std::string&, int, int, size_t, bool, int64_t>(), py::arg("path"), py::arg("rank"),
           py::arg("world"), py::arg("slot_bytes"), py::arg("create"), py::arg("timeout_ms"))
      .def(
          "allreduce",
          [](mbx::CpuMailbox& self, int64_t in, int64_t out, size_t nbytes, int dtype) {
            py::gil_scoped_release nogil;
            return self.allreduce(reinterpret_cast<const void*>(in), reinterpret_cast<void*>(out), nbytes, dtype);
          },
          py::arg("inp"), py::arg("out"), py::arg("nbytes"), py::arg("dtype"))
      .def("reset", &mbx::CpuMailbox::reset)
      .def("set_epoch", &mbx::CpuMailbox::set_epoch)
      .def("close", &mbx::CpuMailbox::close)
      .def("epoch", &mbx::CpuMailbox::epoch)
      .def("error", &mbx::CpuMailbox::error)
      .def("error_peer", &mbx::CpuMailbox::error_peer)
      .def("slot_bytes", &mbx::CpuMailbox::slot_bytes);
  m.def("fdx_listen", &mbx::fdx_listen, py::arg("name"));
  m.def(
      "fdx_send",
      [](const std::string& name, int64_t tag, const std::vector<int>& fds, int timeout_ms) {
        py::gil_scoped_release nogil;
        mbx::fdx_send(name, tag, fds, timeout_ms);
      },
      py::arg("name"), py::arg("tag"), py::arg("fds"), py::arg("timeout_ms"));
  m.def(
      "fdx_recv",
      [](int listen_fd, int count, int timeout_ms) {
        py::gil_scoped_release nogil;
        return mbx::fdx_recv(listen_fd, count, timeout_ms);
      },
      py::arg("listen_fd"), py::arg("count"), py::arg("timeout_ms"));
  m.def("fdx_close", &mbx::fdx_close, py::arg("fd"));
}
