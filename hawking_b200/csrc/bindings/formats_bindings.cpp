// Bindings for the artifact formats (.gravity shards, HGRAV* mixed codecs, sha256, canonical JSON).
#include <pybind11/pybind11.h>
namespace py = pybind11;
void bind_formats(py::module_& m) { (void)m; }
