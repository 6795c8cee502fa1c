/* Host fast path of StreamingGuard.step for one-token ticks (CPython extension module _hsg_host).
 *
 * The reference's step (src/hs_guard/runtime.py:161-174) validates every request in Python, packs the tick
 * (engine/slot_engine_v7.py:117-136, pack_inputs) and builds one result dict per request. For the serving shape
 * in which every request is (int slot, [one int token id]) these three loops are the host's share of a step;
 * here they run in C over the request list:
 *
 *   pack_tokens(requests, max_slots, vocab, hin, nb, length, slots_out) -> n or -1
 *       checks every request against the reference's rules (slot an int in [0, max_slots), unique, ids a
 *       one-element list of an int in [0, vocab)) and writes the lb = 1 packed layout of pack_inputs into hin
 *       (int64 [4 * nb]: ids | lens | slots (padding rows: the scratch slot max_slots) | starts = length[slot]),
 *       and the slots into slots_out. Anything else -- a multi-token request, an int subclass, a tuple of ids,
 *       and every invalid input -- returns -1 before any state changes, and the caller takes the general path,
 *       whose Python validation raises the reference's own error for invalid input.
 *   advance(length, slots, n)              length[slots[i]] += 1 for the n rows of a finished tick
 *   results_single(requests, probs, role, n, nb, tau) -> [{'slot', 'cut_scores', 'threshold'}]
 *       cut score = 1 - p(safe) in float32 (as the reference's 1 - p[:, 0] on a float32 tensor), from the
 *       engine's host output probs (float32 [roles][nb][1][3]); 'slot' is the request's own slot object and
 *       'threshold' the caller's tau object, as in the reference's list.
 *
 * Host code only: no CUDA, no device state.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>
#include <string.h>

static PyObject *k_slot, *k_cut, *k_thr;

/* A C-contiguous buffer of at least `count` items of `itemsize` bytes. */
static int get_buf(PyObject* o, Py_buffer* b, int writable, Py_ssize_t itemsize, Py_ssize_t count, const char* what) {
  if (PyObject_GetBuffer(o, b, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT | (writable ? PyBUF_WRITABLE : 0)) < 0) return -1;
  if (b->itemsize != itemsize || b->len < itemsize * count) {
    PyBuffer_Release(b);
    PyErr_Format(PyExc_ValueError, "%s: need %zd items of %zd bytes", what, count, itemsize);
    return -1;
  }
  return 0;
}

/* (slot, ids) of a request that is an exact 2-tuple or 2-list; 0 if it is neither. */
static int unpack_pair(PyObject* r, PyObject** s, PyObject** ids) {
  if (PyTuple_CheckExact(r) && PyTuple_GET_SIZE(r) == 2) {
    *s = PyTuple_GET_ITEM(r, 0);
    *ids = PyTuple_GET_ITEM(r, 1);
    return 1;
  }
  if (PyList_CheckExact(r) && PyList_GET_SIZE(r) == 2) {
    *s = PyList_GET_ITEM(r, 0);
    *ids = PyList_GET_ITEM(r, 1);
    return 1;
  }
  return 0;
}

/* An exact int in [0, bound), or -1. */
static long long small_int(PyObject* o, long long bound) {
  if (!PyLong_CheckExact(o)) return -1;
  int overflow = 0;
  const long long v = PyLong_AsLongLongAndOverflow(o, &overflow);
  if (overflow || v < 0 || v >= bound) return -1;
  return v;
}

static PyObject* pack_tokens(PyObject* self, PyObject* args) {
  PyObject *requests, *hin_o, *len_o, *slots_o;
  long long max_slots, vocab;
  Py_ssize_t nb;
  if (!PyArg_ParseTuple(args, "OLLOnOO", &requests, &max_slots, &vocab, &hin_o, &nb, &len_o, &slots_o)) return NULL;
  if (!PyList_CheckExact(requests) || max_slots < 1 || vocab < 1) return PyLong_FromLong(-1);
  const Py_ssize_t n = PyList_GET_SIZE(requests);
  if (n == 0 || n > nb) return PyLong_FromLong(-1);
  Py_buffer hb, lb, sb;
  if (get_buf(hin_o, &hb, 1, 8, 4 * nb, "hin") < 0) return NULL;
  if (get_buf(len_o, &lb, 0, 8, max_slots, "length") < 0) {
    PyBuffer_Release(&hb);
    return NULL;
  }
  if (get_buf(slots_o, &sb, 1, 8, n, "slots_out") < 0) {
    PyBuffer_Release(&hb);
    PyBuffer_Release(&lb);
    return NULL;
  }
  unsigned char* seen = (unsigned char*)PyMem_Calloc((size_t)max_slots, 1);
  if (!seen) {
    PyBuffer_Release(&hb);
    PyBuffer_Release(&lb);
    PyBuffer_Release(&sb);
    return PyErr_NoMemory();
  }
  int64_t* ids = (int64_t*)hb.buf;
  int64_t* lens = ids + nb;
  int64_t* sl = ids + 2 * nb;
  int64_t* st = ids + 3 * nb;
  const int64_t* length = (const int64_t*)lb.buf;
  int64_t* out = (int64_t*)sb.buf;
  Py_ssize_t i;
  for (i = 0; i < n; ++i) {
    PyObject *s, *tok;
    if (!unpack_pair(PyList_GET_ITEM(requests, i), &s, &tok)) break;
    const long long sv = small_int(s, max_slots);
    if (sv < 0 || seen[sv]) break;
    seen[sv] = 1;
    if (!PyList_CheckExact(tok) || PyList_GET_SIZE(tok) != 1) break;
    const long long tv = small_int(PyList_GET_ITEM(tok, 0), vocab);
    if (tv < 0) break;
    ids[i] = tv;
    lens[i] = 1;
    sl[i] = sv;
    st[i] = length[sv];
    out[i] = sv;
  }
  const int fast = i == n;
  if (fast) {
    for (; i < nb; ++i) {
      ids[i] = 0;
      lens[i] = 0;
      sl[i] = max_slots;
      st[i] = 0;
    }
  }
  PyMem_Free(seen);
  PyBuffer_Release(&hb);
  PyBuffer_Release(&lb);
  PyBuffer_Release(&sb);
  return PyLong_FromSsize_t(fast ? n : -1);
}

static PyObject* advance(PyObject* self, PyObject* args) {
  PyObject *len_o, *slots_o;
  Py_ssize_t n;
  if (!PyArg_ParseTuple(args, "OOn", &len_o, &slots_o, &n)) return NULL;
  Py_buffer lb, sb;
  if (PyObject_GetBuffer(len_o, &lb, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT | PyBUF_WRITABLE) < 0) return NULL;
  if (lb.itemsize != 8) {
    PyBuffer_Release(&lb);
    PyErr_SetString(PyExc_ValueError, "length: need int64");
    return NULL;
  }
  if (get_buf(slots_o, &sb, 0, 8, n, "slots") < 0) {
    PyBuffer_Release(&lb);
    return NULL;
  }
  int64_t* length = (int64_t*)lb.buf;
  const int64_t* sl = (const int64_t*)sb.buf;
  const Py_ssize_t m = lb.len / 8;
  int bad = 0;
  for (Py_ssize_t i = 0; i < n; ++i) {
    if (sl[i] < 0 || sl[i] >= m) {
      bad = 1;
      break;
    }
  }
  if (!bad)
    for (Py_ssize_t i = 0; i < n; ++i) length[sl[i]] += 1;
  PyBuffer_Release(&lb);
  PyBuffer_Release(&sb);
  if (bad) {
    PyErr_SetString(PyExc_IndexError, "slot outside the length array");
    return NULL;
  }
  Py_RETURN_NONE;
}

static PyObject* results_single(PyObject* self, PyObject* args) {
  PyObject *requests, *probs_o, *tau;
  int role;
  Py_ssize_t n, nb;
  if (!PyArg_ParseTuple(args, "OOinnO", &requests, &probs_o, &role, &n, &nb, &tau)) return NULL;
  if (!PyList_CheckExact(requests) || PyList_GET_SIZE(requests) < n || role < 0) {
    PyErr_SetString(PyExc_ValueError, "results_single: bad arguments");
    return NULL;
  }
  Py_buffer pb;
  if (get_buf(probs_o, &pb, 0, 4, ((Py_ssize_t)role + 1) * nb * 3, "probs") < 0) return NULL;
  const float* p = (const float*)pb.buf + (Py_ssize_t)role * nb * 3;
  PyObject* list = PyList_New(n);
  if (!list) {
    PyBuffer_Release(&pb);
    return NULL;
  }
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject *s, *ids;
    if (!unpack_pair(PyList_GET_ITEM(requests, i), &s, &ids)) {
      PyErr_SetString(PyExc_ValueError, "results_single: request is not a (slot, ids) pair");
      goto fail;
    }
    const float cut = 1.0f - p[i * 3];
    PyObject* c = PyFloat_FromDouble((double)cut);
    if (!c) goto fail;
    PyObject* cl = PyList_New(1);
    if (!cl) {
      Py_DECREF(c);
      goto fail;
    }
    PyList_SET_ITEM(cl, 0, c);
    PyObject* d = PyDict_New();
    if (!d || PyDict_SetItem(d, k_slot, s) < 0 || PyDict_SetItem(d, k_cut, cl) < 0 ||
        PyDict_SetItem(d, k_thr, tau) < 0) {
      Py_XDECREF(d);
      Py_DECREF(cl);
      goto fail;
    }
    Py_DECREF(cl);
    PyList_SET_ITEM(list, i, d);
  }
  PyBuffer_Release(&pb);
  return list;
fail:
  PyBuffer_Release(&pb);
  Py_DECREF(list);
  return NULL;
}

static PyMethodDef methods[] = {
    {"pack_tokens", pack_tokens, METH_VARARGS, "Validate one-token requests and write the lb = 1 packed tick."},
    {"advance", advance, METH_VARARGS, "length[slots[i]] += 1 for i < n."},
    {"results_single", results_single, METH_VARARGS, "The reference's result list for a one-token tick."},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_hsg_host", NULL, -1, methods, NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__hsg_host(void) {
  k_slot = PyUnicode_InternFromString("slot");
  k_cut = PyUnicode_InternFromString("cut_scores");
  k_thr = PyUnicode_InternFromString("threshold");
  if (!k_slot || !k_cut || !k_thr) return NULL;
  return PyModule_Create(&module);
}
