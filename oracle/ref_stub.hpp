// Minimal stand-ins that let the reference's own native headers
// (neuralzip/native/common.h, mixed_huffman.h, gpu_layout.h) compile outside
// a Python extension. TEST INFRASTRUCTURE ONLY: used by oracle/ref_shim.cpp,
// which oracle/Makefile builds into oracle/_ref/libnzref.so from the
// reference sources where they lie. Nothing here is called at run time
// except the trivial buffer/handle plumbing; the Python, nanobind and zstd
// entry points the headers mention are declared but never reached by the
// shim's code paths.
#pragma once

#include <algorithm>
#include <array>
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <exception>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

typedef long Py_ssize_t;
struct StubObject {
    const void* data;
    Py_ssize_t size;
};
typedef StubObject PyObject;
struct Py_buffer {
    void* buf = nullptr;
    Py_ssize_t len = 0;
    PyObject* obj = nullptr;
};
#define PyBUF_CONTIG_RO 0
inline int PyObject_GetBuffer(PyObject* o, Py_buffer* view, int) {
    view->buf = const_cast<void*>(o->data);
    view->len = o->size;
    view->obj = o;
    return 0;
}
inline void PyBuffer_Release(Py_buffer* view) { view->obj = nullptr; }
inline unsigned long long PyLong_AsUnsignedLongLong(PyObject*) { return 0; }
inline PyObject* PyErr_Occurred() { return nullptr; }

namespace stub_nb {
struct handle {
    PyObject* p = nullptr;
    handle() = default;
    handle(PyObject* x) : p(x) {}
    PyObject* ptr() const { return p; }
    bool is_none() const { return p == nullptr; }
};
struct object : handle {};
struct python_error : std::exception {};
using builtin_exception = std::runtime_error;
struct capsule : object {
    void* data(const char*) const { return nullptr; }
};
template <class T>
T borrow(handle h) {
    T t;
    t.p = h.p;
    return t;
}
struct bytes : object {
    bytes(const void*, size_t) {}
};
struct tuple : object {
    tuple() = default;
    explicit tuple(handle) {}
    const handle* begin() const { return nullptr; }
    const handle* end() const { return nullptr; }
    size_t size() const { return 0; }
    handle operator[](size_t) const { return handle(); }
};
struct list : object {
    template <class T>
    void append(T&&) {}
};
struct gil_scoped_release {};
template <class... A>
tuple make_tuple(A&&...) {
    return tuple();
}
}  // namespace stub_nb

#define HUF_BLOCKSIZE_MAX (128 * 1024)
#define HUF_SYMBOLVALUE_MAX 255
#define HUF_TABLELOG_DEFAULT 11
#define HUF_TABLELOG_ABSOLUTEMAX 12
#define DYNAMIC_BMI2 0
#define HUF_flags_disableAsm 1
#define HUF_flags_bmi2 2
typedef size_t HUF_CElt;
typedef uint32_t HUF_DTable;
inline unsigned HUF_isError(size_t) { return 0; }
inline const char* HUF_getErrorName(size_t) { return ""; }
inline int ZSTD_cpuSupportsBmi2() { return 0; }
