// Bindings for the engine host logic (paged-KV block manager, scheduler, n-gram drafter, server).
#include <pybind11/pybind11.h>
namespace py = pybind11;
void bind_engine(py::module_& m) { (void)m; }
