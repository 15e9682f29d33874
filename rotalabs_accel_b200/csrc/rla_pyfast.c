/* CPython fast-call bindings of the hot C-ABI entry points.
 *
 * ctypes converts and checks every argument of every call through generic
 * Python machinery (about 10 us for the 16 arguments of rla_w8a16_gemm on
 * the GPU box's host), more than a decode GEMM takes on the GPU.  This module
 * passes the same plain integers (pointers, strides, sizes, dtype codes, the
 * stream) straight to the library with METH_FASTCALL.  It adds no logic: the
 * arguments, their meaning and the returned status are exactly those of
 * include/rla_w8a16.h; pointers are Python ints (0 = NULL).
 *
 * Built by rotalabs_accel_b200/build.py next to librla_w8a16.so and linked to
 * it (rpath $ORIGIN), so the library state (error string, launch counter,
 * decode-kernel choice) is the one the ctypes bindings see.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

#include "../../include/rla_w8a16.h"

static int get_u64(PyObject* o, unsigned long long* v) {
  *v = PyLong_AsUnsignedLongLong(o);
  return !(*v == (unsigned long long)-1 && PyErr_Occurred());
}

static int get_i64(PyObject* o, long long* v) {
  *v = PyLong_AsLongLong(o);
  return !(*v == -1 && PyErr_Occurred());
}

#define PTR(i) ((void*)(uintptr_t)u[i])

/* gemm(x, ldx, w, ldw, scale, scale_dtype, bias, bias_dtype, y, ldy, M, N, K,
 *      workspace, workspace_bytes, stream) -> status        (rla_w8a16_gemm) */
static PyObject* fast_gemm(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 16) {
    PyErr_SetString(PyExc_TypeError, "gemm expects 16 integer arguments");
    return NULL;
  }
  unsigned long long u[16];
  long long s[16];
  /* pointers and sizes: 0 x, 2 w, 4 scale, 6 bias, 8 y, 13 workspace,
   * 14 workspace_bytes, 15 stream; signed: strides, dtypes, M, N, K */
  static const int is_ptr[16] = {1, 0, 1, 0, 1, 0, 1, 0, 1, 0, 0, 0, 0, 1, 1, 1};
  for (int i = 0; i < 16; ++i) {
    if (is_ptr[i] ? !get_u64(args[i], &u[i]) : !get_i64(args[i], &s[i])) return NULL;
  }
  const int st = rla_w8a16_gemm(PTR(0), s[1], (const int8_t*)PTR(2), s[3], PTR(4), (int)s[5], PTR(6), (int)s[7],
                                PTR(8), s[9], s[10], s[11], s[12], PTR(13), (size_t)u[14], PTR(15));
  return PyLong_FromLong(st);
}

/* gemm_swiglu(x, ldx, w_gate, w_up, ldw, scale_gate, scale_up, scale_dtype,
 *             bias_gate, bias_up, bias_dtype, y, ldy, M, N, K, workspace,
 *             workspace_bytes, stream) -> status          (rla_w8a16_gemm_swiglu) */
static PyObject* fast_gemm_swiglu(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 19) {
    PyErr_SetString(PyExc_TypeError, "gemm_swiglu expects 19 integer arguments");
    return NULL;
  }
  unsigned long long u[19];
  long long s[19];
  static const int is_ptr[19] = {1, 0, 1, 1, 0, 1, 1, 0, 1, 1, 0, 1, 0, 0, 0, 0, 1, 1, 1};
  for (int i = 0; i < 19; ++i) {
    if (is_ptr[i] ? !get_u64(args[i], &u[i]) : !get_i64(args[i], &s[i])) return NULL;
  }
  const int st = rla_w8a16_gemm_swiglu(PTR(0), s[1], (const int8_t*)PTR(2), (const int8_t*)PTR(3), s[4], PTR(5),
                                       PTR(6), (int)s[7], PTR(8), PTR(9), (int)s[10], PTR(11), s[12], s[13], s[14],
                                       s[15], PTR(16), (size_t)u[17], PTR(18));
  return PyLong_FromLong(st);
}

/* workspace_size(M, N, K) -> bytes                     (rla_w8a16_workspace_size) */
static PyObject* fast_workspace_size(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  long long v[3];
  if (nargs != 3) {
    PyErr_SetString(PyExc_TypeError, "workspace_size expects 3 integer arguments");
    return NULL;
  }
  for (int i = 0; i < 3; ++i)
    if (!get_i64(args[i], &v[i])) return NULL;
  return PyLong_FromSize_t(rla_w8a16_workspace_size(v[0], v[1], v[2]));
}

static PyMethodDef methods[] = {
    {"gemm", (PyCFunction)(void (*)(void))fast_gemm, METH_FASTCALL, "rla_w8a16_gemm with integer arguments"},
    {"gemm_swiglu", (PyCFunction)(void (*)(void))fast_gemm_swiglu, METH_FASTCALL,
     "rla_w8a16_gemm_swiglu with integer arguments"},
    {"workspace_size", (PyCFunction)(void (*)(void))fast_workspace_size, METH_FASTCALL,
     "rla_w8a16_workspace_size"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_rla_fast", "Fast-call bindings of librla_w8a16", -1,
                                    methods, NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__rla_fast(void) { return PyModule_Create(&module); }
