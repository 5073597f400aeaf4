/*
 * gw_pyfast.c -- CPython fast-call bindings of the hot C-ABI entry points.
 *
 * The C ABI (include/ghostweight_b200.h) is bound from Python with ctypes,
 * which costs a few microseconds per call to convert every argument. A layer
 * call issues two or three entry points, so at small batch sizes this host
 * time, not the GPU, decided the speed. This module exposes the same entry
 * points as METH_FASTCALL functions that take the arguments as Python ints
 * (device pointers as ints, None for NULL) and return the gw_status int. It
 * calls into libghostweight_b200.so (linked with an $ORIGIN run path, so the
 * one copy that ctypes also loads) and holds no state of its own.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include "ghostweight_b200.h"

/* Argument kinds of one entry point: 'p' pointer (int or None), 'i' int,
 * 'l' int64, 'z' size_t, 'd' double. */
#define GW_MAX_ARGS 20

typedef union {
  void* p;
  int i;
  long long l;
  size_t z;
  double d;
} gw_arg;

static int parse(const char* kinds, PyObject* const* args, Py_ssize_t nargs, gw_arg* out) {
  const Py_ssize_t want = (Py_ssize_t)strlen(kinds);
  if (nargs != want) {
    PyErr_Format(PyExc_TypeError, "expected %zd arguments, got %zd", want, nargs);
    return -1;
  }
  for (Py_ssize_t k = 0; k < nargs; ++k) {
    PyObject* o = args[k];
    switch (kinds[k]) {
      case 'p':
        if (o == Py_None) {
          out[k].p = NULL;
        } else {
          out[k].p = PyLong_AsVoidPtr(o);
          if (out[k].p == NULL && PyErr_Occurred()) return -1;
        }
        break;
      case 'i': {
        const long v = PyLong_AsLong(o);
        if (v == -1 && PyErr_Occurred()) return -1;
        out[k].i = (int)v;
        break;
      }
      case 'l':
        out[k].l = PyLong_AsLongLong(o);
        if (out[k].l == -1 && PyErr_Occurred()) return -1;
        break;
      case 'z':
        out[k].z = PyLong_AsSize_t(o);
        if (out[k].z == (size_t)-1 && PyErr_Occurred()) return -1;
        break;
      case 'd':
        out[k].d = PyFloat_AsDouble(o);
        if (out[k].d == -1.0 && PyErr_Occurred()) return -1;
        break;
      default:
        PyErr_SetString(PyExc_SystemError, "bad argument kind");
        return -1;
    }
  }
  return 0;
}

#define GW_PARSE(KINDS)                                   \
  gw_arg a[GW_MAX_ARGS];                                  \
  if (parse(KINDS, args, nargs, a) < 0) return NULL;

static PyObject* fast_gather_gemm(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("pilllpllplpiplipzp")
  return PyLong_FromLong(gw_gather_gemm(a[0].p, a[1].i, a[2].l, a[3].l, a[4].l, a[5].p, a[6].l,
                                        a[7].l, (const int64_t*)a[8].p, a[9].l, a[10].p, a[11].i,
                                        a[12].p, a[13].l, a[14].i, a[15].p, a[16].z, a[17].p));
}

static PyObject* fast_gather_gemm_dev(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("pilllpllplppiplpzp")
  return PyLong_FromLong(gw_gather_gemm_dev(a[0].p, a[1].i, a[2].l, a[3].l, a[4].l, a[5].p, a[6].l,
                                            a[7].l, (const int64_t*)a[8].p, a[9].l,
                                            (const int32_t*)a[10].p, a[11].p, a[12].i, a[13].p,
                                            a[14].l, a[15].p, a[16].z, a[17].p));
}

static PyObject* fast_packed_gemm(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("pilllpllpiplp")
  return PyLong_FromLong(gw_packed_gemm(a[0].p, a[1].i, a[2].l, a[3].l, a[4].l, a[5].p, a[6].l,
                                        a[7].l, a[8].p, a[9].i, a[10].p, a[11].l, a[12].p));
}

static PyObject* fast_gather_columns(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("pilllplpllp")
  return PyLong_FromLong(gw_gather_columns(a[0].p, a[1].i, a[2].l, a[3].l, a[4].l,
                                           (const int64_t*)a[5].p, a[6].l, a[7].p, a[8].l, a[9].l,
                                           a[10].p));
}

static PyObject* fast_gather_rows_t(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("pilllplpllp")
  return PyLong_FromLong(gw_gather_rows_t(a[0].p, a[1].i, a[2].l, a[3].l, a[4].l,
                                          (const int64_t*)a[5].p, a[6].l, a[7].p, a[8].l, a[9].l,
                                          a[10].p));
}

static PyObject* fast_gather_columns_dev(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("pilllplppllp")
  return PyLong_FromLong(gw_gather_columns_dev(a[0].p, a[1].i, a[2].l, a[3].l, a[4].l,
                                               (const int64_t*)a[5].p, a[6].l,
                                               (const int32_t*)a[7].p, a[8].p, a[9].l, a[10].l,
                                               a[11].p));
}

static PyObject* fast_gather_rows_t_dev(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("pilllplppllp")
  return PyLong_FromLong(gw_gather_rows_t_dev(a[0].p, a[1].i, a[2].l, a[3].l, a[4].l,
                                              (const int64_t*)a[5].p, a[6].l,
                                              (const int32_t*)a[7].p, a[8].p, a[9].l, a[10].l,
                                              a[11].p));
}

static PyObject* fast_mask_compact(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("pillldppppzp")
  return PyLong_FromLong(gw_mask_compact(a[0].p, a[1].i, a[2].l, a[3].l, a[4].l, a[5].d,
                                         (int32_t*)a[6].p, (int64_t*)a[7].p, (int32_t*)a[8].p,
                                         a[9].p, a[10].z, a[11].p));
}

static PyObject* fast_dynamic_linear(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("pilllplldpiplppp")
  return PyLong_FromLong(gw_dynamic_linear(a[0].p, a[1].i, a[2].l, a[3].l, a[4].l, a[5].p, a[6].l,
                                           a[7].l, a[8].d, a[9].p, a[10].i, a[11].p, a[12].l,
                                           (int32_t*)a[13].p, (int32_t*)a[14].p, a[15].p));
}

static PyObject* fast_gather_gemm_workspace_bytes(PyObject* self, PyObject* const* args,
                                                  Py_ssize_t nargs) {
  (void)self;
  GW_PARSE("lli")
  return PyLong_FromSize_t(gw_gather_gemm_workspace_bytes(a[0].l, a[1].l, a[2].i));
}

/* Address of gw_version as this module sees it: lets the loader check that the
 * module and the ctypes binding use one copy of the library. */
static PyObject* fast_library_anchor(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  (void)args;
  if (nargs != 0) {
    PyErr_SetString(PyExc_TypeError, "no arguments expected");
    return NULL;
  }
  return PyLong_FromVoidPtr((void*)&gw_version);
}

#define GW_FAST(name) {#name, (PyCFunction)(void (*)(void))fast_##name, METH_FASTCALL, NULL}
static PyMethodDef gw_fast_methods[] = {
    GW_FAST(gather_gemm),
    GW_FAST(gather_gemm_dev),
    GW_FAST(packed_gemm),
    GW_FAST(gather_columns),
    GW_FAST(gather_rows_t),
    GW_FAST(gather_columns_dev),
    GW_FAST(gather_rows_t_dev),
    GW_FAST(mask_compact),
    GW_FAST(dynamic_linear),
    GW_FAST(gather_gemm_workspace_bytes),
    GW_FAST(library_anchor),
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef gw_fast_module = {
    PyModuleDef_HEAD_INIT, "_gwfast",
    "Fast-call bindings of libghostweight_b200.so's hot entry points (ints in, gw_status out).",
    -1, gw_fast_methods, NULL, NULL, NULL, NULL,
};

PyMODINIT_FUNC PyInit__gwfast(void) { return PyModule_Create(&gw_fast_module); }
