/* CPython module light_vllm_b200._hostpack: reads one step's attention
 * metadata out of its Python objects into flat C arrays for
 * lvb_pack_step_metadata.
 *
 * PagedAttentionMetadata (runtime/execution/paged_attention.py:18-95) holds
 * its block tables as tuples of Python ints and its query layouts as objects
 * with a `parent_indices` tuple.  A decode step of 64 requests at a few
 * thousand tokens of context carries ~10^4 block ids; turning them into an
 * int32 array through numpy costs ~200-300 us per step, longer than the
 * attention kernel itself.  This module walks the objects once with the C API.
 *
 * gather_step(tables, computed, layouts, reserved, readonly,
 *             ids_addr, ids_capacity, offsets_addr, rows_addr)
 *   writes  ids[total]        int32 block ids, rows concatenated (an id that
 *                             does not fit int32 is written as -1, which the
 *                             validator reports as out of range, as the
 *                             reference reports any id >= num_blocks)
 *           offsets[n + 1]    int64 row starts in ids
 *           rows[4 n]         int32: computed | query lengths | reserved |
 *                             readonly prefix blocks
 *   returns (total_ids, max_blocks, num_tokens, max_query_len, max_seq_len,
 *            linear, num_single), linear = every layout is the causal chain,
 *            num_single = requests with one query token
 *            (-1, 0, 1, ..., len - 2).
 * Counts that do not fit int32 raise OverflowError; ids_capacity too small
 * raises ValueError.  The caller owns the buffers (sizes n + 1, 4 n and
 * ids_capacity elements).
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

static PyObject *parent_indices_name;

static int to_i32(PyObject *o, int32_t *out, int clamp) {
#if PY_VERSION_HEX >= 0x030C0000
  /* Exact ints of one machine digit (every block id and count in practice). */
  if (PyLong_CheckExact(o) && PyUnstable_Long_IsCompact((PyLongObject *)o)) {
    const Py_ssize_t v = PyUnstable_Long_CompactValue((PyLongObject *)o);
    if (v >= INT32_MIN && v <= INT32_MAX) {
      *out = (int32_t)v;
      return 0;
    }
  }
#endif
  int overflow = 0;
  long long v = PyLong_AsLongLongAndOverflow(o, &overflow);
  if (v == -1 && PyErr_Occurred()) return -1;
  if (overflow || v > INT32_MAX || v < INT32_MIN) {
    if (clamp) {
      *out = -1;
      return 0;
    }
    PyErr_SetString(PyExc_OverflowError, "step metadata count does not fit int32");
    return -1;
  }
  *out = (int32_t)v;
  return 0;
}

/* Fills dst[0..n) from a sequence of n ints; -1 with an exception set on error. */
static int row_values(PyObject *seq, Py_ssize_t n, int32_t *dst, const char *what) {
  PyObject *fast = PySequence_Fast(seq, what);
  if (!fast) return -1;
  if (PySequence_Fast_GET_SIZE(fast) != n) {
    Py_DECREF(fast);
    PyErr_Format(PyExc_ValueError, "%s must have one entry per request", what);
    return -1;
  }
  PyObject **items = PySequence_Fast_ITEMS(fast);
  for (Py_ssize_t i = 0; i < n; ++i) {
    if (to_i32(items[i], &dst[i], 0) < 0) {
      Py_DECREF(fast);
      return -1;
    }
  }
  Py_DECREF(fast);
  return 0;
}

/* 1 if layout.parent_indices is (-1, 0, ..., len - 2), 0 if not, -1 on error. */
static int is_linear(PyObject *layout) {
  PyObject *parents = PyObject_GetAttr(layout, parent_indices_name);
  if (!parents) return -1;
  PyObject *fast = PySequence_Fast(parents, "parent_indices");
  Py_DECREF(parents);
  if (!fast) return -1;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(fast);
  PyObject **items = PySequence_Fast_ITEMS(fast);
  int linear = 1;
  for (Py_ssize_t j = 0; j < n && linear; ++j) {
    int overflow = 0;
    long long v = PyLong_AsLongLongAndOverflow(items[j], &overflow);
    if (v == -1 && PyErr_Occurred()) {
      Py_DECREF(fast);
      return -1;
    }
    linear = !overflow && v == (long long)j - 1;
  }
  Py_DECREF(fast);
  return linear;
}

static PyObject *gather_step(PyObject *self, PyObject *args) {
  (void)self;
  PyObject *tables, *computed, *layouts, *reserved, *readonly;
  unsigned long long ids_addr, offsets_addr, rows_addr;
  Py_ssize_t ids_capacity;
  if (!PyArg_ParseTuple(args, "OOOOOKnKK", &tables, &computed, &layouts, &reserved, &readonly, &ids_addr,
                        &ids_capacity, &offsets_addr, &rows_addr))
    return NULL;
  int32_t *ids = (int32_t *)(uintptr_t)ids_addr;
  int64_t *offsets = (int64_t *)(uintptr_t)offsets_addr;
  int32_t *rows = (int32_t *)(uintptr_t)rows_addr;

  PyObject *tfast = PySequence_Fast(tables, "block_tables");
  if (!tfast) return NULL;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(tfast);
  PyObject **trows = PySequence_Fast_ITEMS(tfast);
  PyObject *lfast = NULL;
  Py_ssize_t total = 0, max_blocks = 0;
  long long num_tokens = 0, max_query = 0, max_seq = 0, single = 0;
  int linear = 1;

  offsets[0] = 0;
  for (Py_ssize_t r = 0; r < n; ++r) {
    PyObject *row = PySequence_Fast(trows[r], "block table");
    if (!row) goto fail;
    const Py_ssize_t len = PySequence_Fast_GET_SIZE(row);
    if (total + len > ids_capacity) {
      Py_DECREF(row);
      PyErr_SetString(PyExc_ValueError, "block-id buffer is smaller than the block tables");
      goto fail;
    }
    PyObject **items = PySequence_Fast_ITEMS(row);
    for (Py_ssize_t i = 0; i < len; ++i) {
      if (to_i32(items[i], &ids[total + i], 1) < 0) {
        Py_DECREF(row);
        goto fail;
      }
    }
    Py_DECREF(row);
    total += len;
    offsets[r + 1] = total;
    if (len > max_blocks) max_blocks = len;
  }

  int32_t *comp = rows, *qlen = rows + n, *res = rows + 2 * n, *ro = rows + 3 * n;
  if (row_values(computed, n, comp, "num_computed_tokens") < 0) goto fail;
  if (row_values(reserved, n, res, "num_reserved_query_tokens") < 0) goto fail;
  if (row_values(readonly, n, ro, "num_readonly_prefix_blocks") < 0) goto fail;
  lfast = PySequence_Fast(layouts, "query_layouts");
  if (!lfast) goto fail;
  if (PySequence_Fast_GET_SIZE(lfast) != n) {
    PyErr_SetString(PyExc_ValueError, "query_layouts must have one entry per request");
    goto fail;
  }
  PyObject **litems = PySequence_Fast_ITEMS(lfast);
  for (Py_ssize_t r = 0; r < n; ++r) {
    const Py_ssize_t len = PyObject_Size(litems[r]);
    if (len < 0) goto fail;
    if (len > INT32_MAX) {
      PyErr_SetString(PyExc_OverflowError, "step metadata count does not fit int32");
      goto fail;
    }
    qlen[r] = (int32_t)len;
    num_tokens += len;
    single += len == 1;
    if (len > max_query) max_query = len;
    if ((long long)comp[r] + len > max_seq) max_seq = (long long)comp[r] + len;
    if (linear) {
      const int l = is_linear(litems[r]);
      if (l < 0) goto fail;
      linear = l;
    }
  }
  Py_DECREF(lfast);
  Py_DECREF(tfast);
  return Py_BuildValue("(nnLLLOL)", total, max_blocks, num_tokens, max_query, max_seq,
                       linear ? Py_True : Py_False, single);

fail:
  Py_XDECREF(lfast);
  Py_DECREF(tfast);
  return NULL;
}

static PyMethodDef methods[] = {
    {"gather_step", gather_step, METH_VARARGS,
     "gather_step(tables, computed, layouts, reserved, readonly, ids_addr, ids_capacity, offsets_addr, "
     "rows_addr) -> (total_ids, max_blocks, num_tokens, max_query_len, max_seq_len, linear, "
     "num_single)"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef module = {
    PyModuleDef_HEAD_INIT,
    .m_name = "_hostpack",
    .m_doc = "Step-metadata gathering from Python objects into C arrays.",
    .m_size = -1,
    .m_methods = methods,
};

PyMODINIT_FUNC PyInit__hostpack(void) {
  parent_indices_name = PyUnicode_InternFromString("parent_indices");
  if (!parent_indices_name) return NULL;
  return PyModule_Create(&module);
}
