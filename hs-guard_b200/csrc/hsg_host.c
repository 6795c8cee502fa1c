/* Host fast path of StreamingGuard.step for ticks that fit one launch (CPython extension module _hsg_host).
 *
 * The reference's step (src/hs_guard/runtime.py:161-174) validates every request in Python, packs the tick
 * (engine/slot_engine_v7.py:7-25 pack_inputs, :117-136) and builds one result dict per request. For the shapes a
 * server sends -- a list of (int slot, [int token ids]) with unique slots and at most 64 ids each -- these loops are
 * the host's share of a step; here they run in C over the request list:
 *
 *   scan(requests, max_slots, vocab) -> longest request, or -1
 *       the reference's rules (slot an int in [0, max_slots), slots unique, ids a nonempty list of ints in
 *       [0, vocab)) for requests that are exactly that: a list of 2-tuples / 2-lists of exact ints and lists of
 *       exact ints. Anything else -- an int subclass such as bool, a tuple of ids, and every invalid input --
 *       gives -1, and the caller takes the general path, whose Python validation accepts what the reference
 *       accepts and raises the reference's own error otherwise. Nothing is written.
 *   fill(requests, hin, nb, lb, length, max_slots)
 *       pack_inputs' layout into hin (int64 [nb * lb + 3 * nb]): ids [nb][lb] right-padded with 0 | lens |
 *       slots (padding rows: the scratch slot max_slots) | starts = length[slot] (padding rows 0), for requests
 *       that scan accepted with longest <= lb and len(requests) <= nb.
 *   advance(length, hin, nb, lb, n)   length[slot] += len for the n rows of the packed tick (after it ran)
 *   results(requests, probs, role, n, nb, lb, tau) -> [{'slot', 'cut_scores', 'threshold'}]
 *       cut score = 1 - p(safe) per token in float32 (the reference's 1 - p[:, 0] on a float32 tensor) from the
 *       engine's host output probs (float32 [roles][nb][lb][3]); 'slot' is the request's own slot object and
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

static PyObject* scan(PyObject* self, PyObject* args) {
  PyObject* requests;
  long long max_slots, vocab;
  if (!PyArg_ParseTuple(args, "OLL", &requests, &max_slots, &vocab)) return NULL;
  if (!PyList_CheckExact(requests) || max_slots < 1 || vocab < 1) return PyLong_FromLong(-1);
  const Py_ssize_t n = PyList_GET_SIZE(requests);
  if (n == 0) return PyLong_FromLong(-1);
  unsigned char* seen = (unsigned char*)PyMem_Calloc((size_t)max_slots, 1);
  if (!seen) return PyErr_NoMemory();
  Py_ssize_t longest = 0;
  for (Py_ssize_t i = 0; i < n && longest >= 0; ++i) {
    PyObject *s, *ids;
    if (!unpack_pair(PyList_GET_ITEM(requests, i), &s, &ids) || !PyList_CheckExact(ids)) {
      longest = -1;
      break;
    }
    const long long sv = small_int(s, max_slots);
    const Py_ssize_t m = PyList_GET_SIZE(ids);
    if (sv < 0 || seen[sv] || m == 0) {
      longest = -1;
      break;
    }
    seen[sv] = 1;
    for (Py_ssize_t t = 0; t < m; ++t) {
      if (small_int(PyList_GET_ITEM(ids, t), vocab) < 0) {
        longest = -1;
        break;
      }
    }
    if (m > longest && longest >= 0) longest = m;
  }
  PyMem_Free(seen);
  return PyLong_FromSsize_t(longest);
}

static PyObject* fill(PyObject* self, PyObject* args) {
  PyObject *requests, *hin_o, *len_o;
  Py_ssize_t nb, lb;
  long long max_slots;
  if (!PyArg_ParseTuple(args, "OOnnOL", &requests, &hin_o, &nb, &lb, &len_o, &max_slots)) return NULL;
  if (!PyList_CheckExact(requests) || nb < 1 || lb < 1 || PyList_GET_SIZE(requests) > nb) {
    PyErr_SetString(PyExc_ValueError, "fill: the tick does not fit its bucket");
    return NULL;
  }
  const Py_ssize_t n = PyList_GET_SIZE(requests);
  Py_buffer hb, lenb;
  if (get_buf(hin_o, &hb, 1, 8, nb * lb + 3 * nb, "hin") < 0) return NULL;
  if (get_buf(len_o, &lenb, 0, 8, max_slots, "length") < 0) {
    PyBuffer_Release(&hb);
    return NULL;
  }
  int64_t* ids = (int64_t*)hb.buf;
  int64_t* lens = ids + nb * lb;
  int64_t* sl = lens + nb;
  int64_t* st = sl + nb;
  const int64_t* length = (const int64_t*)lenb.buf;
  int bad = 0;
  for (Py_ssize_t i = 0; i < n && !bad; ++i) {
    PyObject *s, *tok;
    if (!unpack_pair(PyList_GET_ITEM(requests, i), &s, &tok) || !PyList_CheckExact(tok)) {
      bad = 1;
      break;
    }
    const long long sv = small_int(s, max_slots);
    const Py_ssize_t m = PyList_GET_SIZE(tok);
    if (sv < 0 || m < 1 || m > lb) {
      bad = 1;
      break;
    }
    int64_t* row = ids + i * lb;
    for (Py_ssize_t t = 0; t < m; ++t) row[t] = PyLong_AsLongLong(PyList_GET_ITEM(tok, t));
    for (Py_ssize_t t = m; t < lb; ++t) row[t] = 0;
    lens[i] = m;
    sl[i] = sv;
    st[i] = length[sv];
  }
  if (!bad) {
    memset(ids + n * lb, 0, (size_t)((nb - n) * lb) * sizeof(int64_t));
    for (Py_ssize_t i = n; i < nb; ++i) {
      lens[i] = 0;
      sl[i] = max_slots;
      st[i] = 0;
    }
  }
  PyBuffer_Release(&hb);
  PyBuffer_Release(&lenb);
  if (bad || PyErr_Occurred()) {
    if (!PyErr_Occurred()) PyErr_SetString(PyExc_ValueError, "fill: requests that scan did not accept");
    return NULL;
  }
  Py_RETURN_NONE;
}

static PyObject* advance(PyObject* self, PyObject* args) {
  PyObject *len_o, *hin_o;
  Py_ssize_t nb, lb, n;
  if (!PyArg_ParseTuple(args, "OOnnn", &len_o, &hin_o, &nb, &lb, &n)) return NULL;
  if (n < 0 || n > nb || lb < 1) {
    PyErr_SetString(PyExc_ValueError, "advance: bad sizes");
    return NULL;
  }
  Py_buffer lenb, hb;
  if (PyObject_GetBuffer(len_o, &lenb, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT | PyBUF_WRITABLE) < 0) return NULL;
  if (lenb.itemsize != 8) {
    PyBuffer_Release(&lenb);
    PyErr_SetString(PyExc_ValueError, "length: need int64");
    return NULL;
  }
  if (get_buf(hin_o, &hb, 0, 8, nb * lb + 3 * nb, "hin") < 0) {
    PyBuffer_Release(&lenb);
    return NULL;
  }
  int64_t* length = (int64_t*)lenb.buf;
  const int64_t* lens = (const int64_t*)hb.buf + nb * lb;
  const int64_t* sl = lens + nb;
  const Py_ssize_t m = lenb.len / 8;
  int bad = 0;
  for (Py_ssize_t i = 0; i < n; ++i) bad |= sl[i] < 0 || sl[i] >= m;
  if (!bad)
    for (Py_ssize_t i = 0; i < n; ++i) length[sl[i]] += lens[i];
  PyBuffer_Release(&lenb);
  PyBuffer_Release(&hb);
  if (bad) {
    PyErr_SetString(PyExc_IndexError, "slot outside the length array");
    return NULL;
  }
  Py_RETURN_NONE;
}

static PyObject* results(PyObject* self, PyObject* args) {
  PyObject *requests, *probs_o, *tau;
  int role;
  Py_ssize_t n, nb, lb;
  if (!PyArg_ParseTuple(args, "OOinnnO", &requests, &probs_o, &role, &n, &nb, &lb, &tau)) return NULL;
  if (!PyList_CheckExact(requests) || PyList_GET_SIZE(requests) < n || n > nb || role < 0 || lb < 1) {
    PyErr_SetString(PyExc_ValueError, "results: bad arguments");
    return NULL;
  }
  Py_buffer pb;
  if (get_buf(probs_o, &pb, 0, 4, ((Py_ssize_t)role + 1) * nb * lb * 3, "probs") < 0) return NULL;
  const float* p = (const float*)pb.buf + (Py_ssize_t)role * nb * lb * 3;
  PyObject* list = PyList_New(n);
  if (!list) {
    PyBuffer_Release(&pb);
    return NULL;
  }
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject *s, *ids;
    if (!unpack_pair(PyList_GET_ITEM(requests, i), &s, &ids) || !PyList_CheckExact(ids) ||
        PyList_GET_SIZE(ids) > lb) {
      PyErr_SetString(PyExc_ValueError, "results: request is not a (slot, ids) pair of the tick");
      goto fail;
    }
    const Py_ssize_t m = PyList_GET_SIZE(ids);
    PyObject* cl = PyList_New(m);
    if (!cl) goto fail;
    for (Py_ssize_t t = 0; t < m; ++t) {
      const float cut = 1.0f - p[(i * lb + t) * 3];
      PyObject* c = PyFloat_FromDouble((double)cut);
      if (!c) {
        Py_DECREF(cl);
        goto fail;
      }
      PyList_SET_ITEM(cl, t, c);
    }
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
    {"scan", scan, METH_VARARGS, "Validate a tick's requests (the reference's rules); longest request or -1."},
    {"fill", fill, METH_VARARGS, "Write pack_inputs' layout of a scanned tick."},
    {"advance", advance, METH_VARARGS, "length[slot] += len for the rows of a packed tick."},
    {"results", results, METH_VARARGS, "The reference's result list of a tick."},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_hsg_host", NULL, -1, methods, NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__hsg_host(void) {
  k_slot = PyUnicode_InternFromString("slot");
  k_cut = PyUnicode_InternFromString("cut_scores");
  k_thr = PyUnicode_InternFromString("threshold");
  if (!k_slot || !k_cut || !k_thr) return NULL;
  return PyModule_Create(&module);
}
