// Minimal CPython binding of the per-call entry point fu_qkv_forward: the
// launch path of FlashUlyssesContext.ulysses_qkv_forward passes 14 plain
// integers/floats per call, which ctypes converts in ~3 us and this
// METH_FASTCALL function in well under 1 us.  Everything else (buffers,
// context creation, errors) stays on the ctypes binding of the same library.
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include "flash_ulysses_b200.h"

namespace {

inline void* as_ptr(PyObject* o) {
    return o == Py_None ? nullptr : PyLong_AsVoidPtr(o);
}

// forward(handle, x, w, positions, q_gamma, k_gamma, rope, local_tokens,
//         rope_rows, q_eps, k_eps, flags, stream, gemm_out) -> None
PyObject* forward(PyObject*, PyObject* const* args, Py_ssize_t nargs) {
    if (nargs != 14) {
        PyErr_SetString(PyExc_TypeError, "forward() takes 14 arguments");
        return nullptr;
    }
    fu_qkv_ctx* ctx = static_cast<fu_qkv_ctx*>(as_ptr(args[0]));
    const void* x = as_ptr(args[1]);
    const void* w = as_ptr(args[2]);
    const int64_t* pos = static_cast<const int64_t*>(as_ptr(args[3]));
    const float* qg = static_cast<const float*>(as_ptr(args[4]));
    const float* kg = static_cast<const float*>(as_ptr(args[5]));
    const float* rope = static_cast<const float*>(as_ptr(args[6]));
    const long long L = PyLong_AsLongLong(args[7]);
    const long long rows = PyLong_AsLongLong(args[8]);
    const double q_eps = PyFloat_AsDouble(args[9]);
    const double k_eps = PyFloat_AsDouble(args[10]);
    const unsigned long flags = PyLong_AsUnsignedLong(args[11]);
    void* stream = as_ptr(args[12]);
    void* gemm_out = as_ptr(args[13]);
    if (PyErr_Occurred()) return nullptr;
    int rc;
    Py_BEGIN_ALLOW_THREADS
    rc = fu_qkv_forward(ctx, x, w, pos, qg, kg, rope, L, rows, q_eps, k_eps,
                        static_cast<uint32_t>(flags), stream, gemm_out);
    Py_END_ALLOW_THREADS
    if (rc != FU_OK) {
        PyErr_Format(PyExc_RuntimeError, "fu_qkv_forward failed (code %d): %s", rc,
                     fu_last_error());
        return nullptr;
    }
    Py_RETURN_NONE;
}

PyMethodDef methods[] = {
    {"forward", reinterpret_cast<PyCFunction>(reinterpret_cast<void (*)()>(forward)),
     METH_FASTCALL, "fu_qkv_forward with plain integer/float arguments"},
    {nullptr, nullptr, 0, nullptr},
};

PyModuleDef module = {PyModuleDef_HEAD_INIT, "_fu_fast", nullptr, -1, methods,
                      nullptr, nullptr, nullptr, nullptr};

}  // namespace

PyMODINIT_FUNC PyInit__fu_fast(void) { return PyModule_Create(&module); }
