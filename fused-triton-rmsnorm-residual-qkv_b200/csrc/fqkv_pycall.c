/* CPython fast path for the hot C-ABI call of the Python package (fqkv_launch).
 *
 * The package binds the library with ctypes; converting fqkv_launch's 22 arguments through
 * ctypes costs a few microseconds per call, more than the C entry point itself (which is
 * mostly the CUDA launch).  This module converts them with the CPython API
 * (METH_FASTCALL) and calls the library's fqkv_launch through a function pointer that the
 * package hands over after loading the library (set_launch), so the library it calls is
 * always the one ctypes loaded.  It has no CUDA or PyTorch dependency of its own.
 *
 * launch(x, residual, rms_weight, rms_weight_dtype, weight, out, residual_out, M, H, N,
 *        ldx, ldr, ldw, ldo, ldro, eps, dtype, schedule, flags, workspace, workspace_bytes,
 *        stream) -> int: the arguments of fqkv_launch in order (pointers and the stream as
 *        Python ints, None for a null pointer); returns its return code. */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

typedef int (*fqkv_launch_fn)(const void*, const void*, const void*, int, const void*, void*, void*, int64_t,
                              int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float, int, int, int,
                              void*, int64_t, void*);

static fqkv_launch_fn g_launch = NULL;

static void* as_ptr(PyObject* o) { return o == Py_None ? NULL : PyLong_AsVoidPtr(o); }

static PyObject* set_launch(PyObject* self, PyObject* arg) {
  (void)self;
  void* p = PyLong_AsVoidPtr(arg);
  if (p == NULL && PyErr_Occurred()) return NULL;
  g_launch = (fqkv_launch_fn)p;
  Py_RETURN_NONE;
}

static PyObject* launch(PyObject* self, PyObject* const* a, Py_ssize_t n) {
  (void)self;
  if (n != 22) {
    PyErr_Format(PyExc_TypeError, "launch takes 22 arguments (%zd given)", n);
    return NULL;
  }
  if (g_launch == NULL) {
    PyErr_SetString(PyExc_RuntimeError, "launch: the library's fqkv_launch has not been set");
    return NULL;
  }
  const void* x = as_ptr(a[0]);
  const void* r = as_ptr(a[1]);
  const void* g = as_ptr(a[2]);
  const int gdt = (int)PyLong_AsLong(a[3]);
  const void* w = as_ptr(a[4]);
  void* out = as_ptr(a[5]);
  void* rout = as_ptr(a[6]);
  int64_t v[8];
  for (int i = 0; i < 8; ++i) v[i] = (int64_t)PyLong_AsLongLong(a[7 + i]); /* M H N ldx ldr ldw ldo ldro */
  const float eps = (float)PyFloat_AsDouble(a[15]);
  const int dtype = (int)PyLong_AsLong(a[16]);
  const int schedule = (int)PyLong_AsLong(a[17]);
  const int flags = (int)PyLong_AsLong(a[18]);
  void* ws = as_ptr(a[19]);
  const int64_t ws_bytes = (int64_t)PyLong_AsLongLong(a[20]);
  void* stream = as_ptr(a[21]);
  if (PyErr_Occurred()) return NULL;
  const int rc = g_launch(x, r, g, gdt, w, out, rout, v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], eps, dtype,
                          schedule, flags, ws, ws_bytes, stream);
  return PyLong_FromLong(rc);
}

static PyMethodDef kMethods[] = {
    {"set_launch", (PyCFunction)set_launch, METH_O, "Set the address of the library's fqkv_launch."},
    {"launch", (PyCFunction)(void (*)(void))launch, METH_FASTCALL, "Call fqkv_launch with 22 arguments."},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_fqkv_pycall", NULL, -1, kMethods,
                                     NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__fqkv_pycall(void) { return PyModule_Create(&kModule); }
