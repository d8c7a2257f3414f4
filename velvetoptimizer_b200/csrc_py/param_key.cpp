// Host helper of the PyTorch modules' repack check: the (data pointer, version) pair of
// every parameter of a list in one call, as bytes (16 per tensor).  The modules compare
// these bytes before each forward to see whether the packed weights are stale; done in
// Python, reading 900 parameters' pointers and versions one attribute at a time costs more
// than a decode-sized forward on the GPU.
#include <Python.h>

#include <cstdint>
#include <cstring>

#include <torch/csrc/autograd/python_variable.h>

namespace {

PyObject* pairs(PyObject*, PyObject* seq) {
  PyObject* fast = PySequence_Fast(seq, "pairs() takes a sequence of tensors");
  if (!fast) return nullptr;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(fast);
  PyObject* out = PyBytes_FromStringAndSize(nullptr, n * 16);
  if (!out) {
    Py_DECREF(fast);
    return nullptr;
  }
  char* buf = PyBytes_AS_STRING(out);
  PyObject** items = PySequence_Fast_ITEMS(fast);
  try {
    for (Py_ssize_t i = 0; i < n; ++i) {
      if (!THPVariable_Check(items[i])) {
        PyErr_SetString(PyExc_TypeError, "pairs() takes a sequence of tensors");
        Py_DECREF(out);
        Py_DECREF(fast);
        return nullptr;
      }
      const at::Tensor& t = THPVariable_Unpack(items[i]);
      const uint64_t v[2] = {static_cast<uint64_t>(reinterpret_cast<uintptr_t>(t.data_ptr())),
                             static_cast<uint64_t>(t._version())};
      std::memcpy(buf + 16 * i, v, 16);
    }
  } catch (const std::exception& e) {
    PyErr_SetString(PyExc_RuntimeError, e.what());
    Py_DECREF(out);
    Py_DECREF(fast);
    return nullptr;
  }
  Py_DECREF(fast);
  return out;
}

PyMethodDef kMethods[] = {
    {"pairs", pairs, METH_O, "(data_ptr, version) of every tensor, 16 bytes each"},
    {nullptr, nullptr, 0, nullptr},
};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_param_key", nullptr, -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__param_key() { return PyModule_Create(&kModule); }
