/*
 * histpack.c -- host-side packing of per-row token histories for ns_sample.
 *
 * The engine hands the sampler its histories as Python lists of ints (prompt +
 * generated ids per row; reference sampler.py:36-91 takes
 * all_generated_ids: List[List[int]]).  ns_sample wants them as one int32
 * CSR array in pinned memory.  Converting ~10^5 - 10^6 Python ints per step
 * with array.array costs ~14 ns per id, more than the logits' own PCIe copy;
 * this loop reads the list items directly.
 *
 *   pack(rows, out) -> n
 *     rows: a sequence of sequences of ints; out: a writable buffer of int32
 *     (e.g. a numpy view of the pinned block).  Writes the ids row after row
 *     and returns how many were written.  An id outside int32 raises
 *     OverflowError; a non-integer raises TypeError; ids past the buffer raise
 *     ValueError.  Nothing is written past out.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

static PyObject* pack(PyObject* self, PyObject* args) {
  (void)self;
  PyObject* rows;
  Py_buffer buf;
  if (!PyArg_ParseTuple(args, "Ow*", &rows, &buf)) return NULL;
  PyObject* seq = PySequence_Fast(rows, "histories must be a sequence of sequences");
  if (!seq) {
    PyBuffer_Release(&buf);
    return NULL;
  }
  int32_t* out = (int32_t*)buf.buf;
  const Py_ssize_t cap = buf.len / (Py_ssize_t)sizeof(int32_t);
  Py_ssize_t pos = 0;
  const Py_ssize_t nrows = PySequence_Fast_GET_SIZE(seq);
  for (Py_ssize_t i = 0; i < nrows; ++i) {
    PyObject* rs = PySequence_Fast(PySequence_Fast_GET_ITEM(seq, i), "each history must be a sequence");
    if (!rs) goto fail;
    const Py_ssize_t n = PySequence_Fast_GET_SIZE(rs);
    if (n > cap - pos) {
      Py_DECREF(rs);
      PyErr_SetString(PyExc_ValueError, "history ids exceed the output buffer");
      goto fail;
    }
    PyObject** items = PySequence_Fast_ITEMS(rs);
    for (Py_ssize_t j = 0; j < n; ++j) {
      PyObject* o = items[j];
      long v;
#if PY_VERSION_HEX >= 0x030C0000
      if (PyLong_CheckExact(o) && PyUnstable_Long_IsCompact((PyLongObject*)o))
        v = (long)PyUnstable_Long_CompactValue((PyLongObject*)o);  /* one-digit ints, read directly */
      else
#endif
        v = PyLong_AsLong(o);
      if (v == -1 && PyErr_Occurred()) {
        Py_DECREF(rs);
        goto fail;
      }
      if (v < INT32_MIN || v > INT32_MAX) {
        Py_DECREF(rs);
        PyErr_SetString(PyExc_OverflowError, "history id outside int32");
        goto fail;
      }
      out[pos++] = (int32_t)v;
    }
    Py_DECREF(rs);
  }
  Py_DECREF(seq);
  PyBuffer_Release(&buf);
  return PyLong_FromSsize_t(pos);
fail:
  Py_DECREF(seq);
  PyBuffer_Release(&buf);
  return NULL;
}

static PyMethodDef methods[] = {
    {"pack", pack, METH_VARARGS, "pack(rows, out) -> n: int32 ids of every row, row after row"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_histpack", NULL, -1, methods,
                                    NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__histpack(void) { return PyModule_Create(&module); }
