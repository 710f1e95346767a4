/* Direct CPython calls into the C ABI for the eviction latency path.
 *
 * The eviction decision (score 16K blocks, select the k lowest) takes
 * ~13 us on the GPU, so the host cost of reaching the launch matters: a
 * ctypes call with 15 converted arguments costs ~2.2 us, this module's
 * METH_FASTCALL functions ~0.2 us.  Each function takes the C ABI
 * entry point's arguments in order -- device pointers and the stream as
 * Python ints (None for a null pointer), sizes as ints, weights as floats
 * -- and returns its status code; pagedkv_fusion._C checks the tensors and
 * raises on a nonzero status exactly as on its ctypes path.  Built by
 * build.py with the host C compiler against this interpreter's headers and
 * linked to libpagedkv_sm100.so beside it.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

#include "pagedkv_fusion.h"

static int as_ptr(PyObject* o, void** out) {
  if (o == Py_None) {
    *out = NULL;
    return 0;
  }
  *out = PyLong_AsVoidPtr(o);
  return (*out == NULL && PyErr_Occurred()) ? -1 : 0;
}

static int as_i64(PyObject* o, int64_t* out) {
  *out = (int64_t)PyLong_AsLongLong(o);
  return (*out == -1 && PyErr_Occurred()) ? -1 : 0;
}

static int as_f32(PyObject* o, float* out) {
  const double d = PyFloat_AsDouble(o);
  if (d == -1.0 && PyErr_Occurred()) return -1;
  *out = (float)d;
  return 0;
}

static int nargs_ok(Py_ssize_t got, Py_ssize_t want, const char* name) {
  if (got == want) return 1;
  PyErr_Format(PyExc_TypeError, "%s takes %zd arguments (%zd given)", name, want, got);
  return 0;
}

/* eviction_scores(rec, freq, attn, valid, out, num_blocks, block_size,
 *                 w_recency, w_frequency, w_attention, stream) */
static PyObject* py_eviction_scores(PyObject* self, PyObject* const* a, Py_ssize_t n) {
  void *rec, *freq, *attn, *valid, *out, *stream;
  int64_t nb, bs;
  float wr, wf, wa;
  (void)self;
  if (!nargs_ok(n, 11, "eviction_scores")) return NULL;
  if (as_ptr(a[0], &rec) || as_ptr(a[1], &freq) || as_ptr(a[2], &attn) || as_ptr(a[3], &valid) ||
      as_ptr(a[4], &out) || as_i64(a[5], &nb) || as_i64(a[6], &bs) || as_f32(a[7], &wr) ||
      as_f32(a[8], &wf) || as_f32(a[9], &wa) || as_ptr(a[10], &stream))
    return NULL;
  return PyLong_FromLong(pkv_eviction_scores((const float*)rec, (const float*)freq,
                                             (const float*)attn, (const uint8_t*)valid,
                                             (float*)out, nb, (int32_t)bs, wr, wf, wa, stream));
}

/* eviction_select(scores, num_blocks, k, out, workspace, workspace_bytes, stream) */
static PyObject* py_eviction_select(PyObject* self, PyObject* const* a, Py_ssize_t n) {
  void *scores, *out, *ws, *stream;
  int64_t nb, k, wsb;
  (void)self;
  if (!nargs_ok(n, 7, "eviction_select")) return NULL;
  if (as_ptr(a[0], &scores) || as_i64(a[1], &nb) || as_i64(a[2], &k) || as_ptr(a[3], &out) ||
      as_ptr(a[4], &ws) || as_i64(a[5], &wsb) || as_ptr(a[6], &stream))
    return NULL;
  return PyLong_FromLong(pkv_eviction_select((const float*)scores, nb, k, (int64_t*)out, ws,
                                             (size_t)wsb, stream));
}

/* eviction_scores_select(rec, freq, attn, valid, scores, num_blocks,
 *   block_size, w_recency, w_frequency, w_attention, k, out, workspace,
 *   workspace_bytes, stream) */
static PyObject* py_eviction_scores_select(PyObject* self, PyObject* const* a, Py_ssize_t n) {
  void *rec, *freq, *attn, *valid, *scores, *out, *ws, *stream;
  int64_t nb, bs, k, wsb;
  float wr, wf, wa;
  (void)self;
  if (!nargs_ok(n, 15, "eviction_scores_select")) return NULL;
  if (as_ptr(a[0], &rec) || as_ptr(a[1], &freq) || as_ptr(a[2], &attn) || as_ptr(a[3], &valid) ||
      as_ptr(a[4], &scores) || as_i64(a[5], &nb) || as_i64(a[6], &bs) || as_f32(a[7], &wr) ||
      as_f32(a[8], &wf) || as_f32(a[9], &wa) || as_i64(a[10], &k) || as_ptr(a[11], &out) ||
      as_ptr(a[12], &ws) || as_i64(a[13], &wsb) || as_ptr(a[14], &stream))
    return NULL;
  return PyLong_FromLong(pkv_eviction_scores_select(
      (const float*)rec, (const float*)freq, (const float*)attn, (const uint8_t*)valid,
      (float*)scores, nb, (int32_t)bs, wr, wf, wa, k, (int64_t*)out, ws, (size_t)wsb, stream));
}

static PyMethodDef kMethods[] = {
    {"eviction_scores", (PyCFunction)(void (*)(void))py_eviction_scores, METH_FASTCALL,
     "pkv_eviction_scores; returns the status code"},
    {"eviction_select", (PyCFunction)(void (*)(void))py_eviction_select, METH_FASTCALL,
     "pkv_eviction_select; returns the status code"},
    {"eviction_scores_select", (PyCFunction)(void (*)(void))py_eviction_scores_select,
     METH_FASTCALL, "pkv_eviction_scores_select; returns the status code"},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_pkv_pycall",
                                     "Direct calls into libpagedkv_sm100.so", -1, kMethods};

PyMODINIT_FUNC PyInit__pkv_pycall(void) { return PyModule_Create(&kModule); }
