/* _hostbuf: host addresses of many Python buffers in one call.
 *
 * addresses(objs, out) writes the data address of every object of the
 * sequence `objs` (bytes, bytearray, memoryview, numpy arrays: anything with
 * a contiguous buffer) into `out`, a writable buffer of len(objs) uint64.
 * Each address is read through the buffer protocol (PyObject_GetBuffer with
 * PyBUF_SIMPLE), which is the documented way to reach an object's bytes; it
 * stays valid while the object lives and is not resized, so callers keep the
 * objects referenced and unchanged until they are done with the addresses.
 * Used by the KV page reload to hand tens of thousands of `.kvz` blobs to
 * the native gather without copying them.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

static PyObject* addresses(PyObject* self, PyObject* args) {
  PyObject* seq;
  Py_buffer out;
  (void)self;
  if (!PyArg_ParseTuple(args, "Ow*", &seq, &out)) return NULL;
  PyObject* fast = PySequence_Fast(seq, "addresses() needs a sequence");
  if (!fast) {
    PyBuffer_Release(&out);
    return NULL;
  }
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(fast);
  if (out.len < (Py_ssize_t)(n * sizeof(uint64_t))) {
    Py_DECREF(fast);
    PyBuffer_Release(&out);
    PyErr_SetString(PyExc_ValueError, "output buffer too small");
    return NULL;
  }
  uint64_t* dst = (uint64_t*)out.buf;
  PyObject** items = PySequence_Fast_ITEMS(fast);
  for (Py_ssize_t i = 0; i < n; i++) {
    Py_buffer b;
    if (PyObject_GetBuffer(items[i], &b, PyBUF_SIMPLE) != 0) {
      Py_DECREF(fast);
      PyBuffer_Release(&out);
      return NULL;
    }
    dst[i] = (uint64_t)(uintptr_t)b.buf;
    PyBuffer_Release(&b);
  }
  Py_DECREF(fast);
  PyBuffer_Release(&out);
  Py_RETURN_NONE;
}

static PyMethodDef methods[] = {
    {"addresses", addresses, METH_VARARGS, "Data addresses of a sequence of buffers."},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_hostbuf", NULL, -1, methods};

PyMODINIT_FUNC PyInit__hostbuf(void) { return PyModule_Create(&module); }
