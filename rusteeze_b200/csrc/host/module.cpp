// Python module for the host-side C++ runtime pieces.
#include <pybind11/pybind11.h>

namespace py = pybind11;

void bind_block_manager(py::module_& m);
void bind_runtime(py::module_& m);
void bind_ngram(py::module_& m);

PYBIND11_MODULE(_host, m) {
  m.doc() = "rusteeze_b200 host runtime: KV block manager, batch builder, staging pool, shm ring, n-gram proposer";
  bind_block_manager(m);
  bind_runtime(m);
  bind_ngram(m);
}
