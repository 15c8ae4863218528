/* CPython module light_vllm_b200._hostpack: reads one step's attention
 * metadata out of its Python objects into flat C arrays for
 * lvb_pack_step_metadata, and calls the attention step's library entry
 * points with C-API argument parsing (call trampolines, below).
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

/* The query count of a layout, len(layout.parent_indices), and when
 * `linear` is given whether the parents are (-1, 0, ..., len - 2).  Returns
 * 0 with an exception set on error. */
static int layout_shape(PyObject *layout, Py_ssize_t *len, int *linear) {
  PyObject *parents = PyObject_GetAttr(layout, parent_indices_name);
  if (!parents) return 0;
  PyObject *fast = PySequence_Fast(parents, "parent_indices");
  Py_DECREF(parents);
  if (!fast) return 0;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(fast);
  *len = n;
  if (linear) {
    PyObject **items = PySequence_Fast_ITEMS(fast);
    int lin = 1;
    for (Py_ssize_t j = 0; j < n && lin; ++j) {
      int overflow = 0;
      long long v = PyLong_AsLongLongAndOverflow(items[j], &overflow);
      if (v == -1 && PyErr_Occurred()) {
        Py_DECREF(fast);
        return 0;
      }
      lin = !overflow && v == (long long)j - 1;
    }
    *linear = lin;
  }
  Py_DECREF(fast);
  return 1;
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
    int32_t *dst = ids + total;
    for (Py_ssize_t i = 0; i < len; ++i) {
#if PY_VERSION_HEX >= 0x030C0000
      /* Inline fast path: exact one-digit ints (every block id in practice). */
      PyObject *o = items[i];
      if (i + 8 < len) __builtin_prefetch(items[i + 8]);
      if (PyLong_CheckExact(o) && PyUnstable_Long_IsCompact((PyLongObject *)o)) {
        const Py_ssize_t v = PyUnstable_Long_CompactValue((PyLongObject *)o);
        dst[i] = v >= INT32_MIN && v <= INT32_MAX ? (int32_t)v : -1;
        continue;
      }
#endif
      if (to_i32(items[i], &dst[i], 1) < 0) {
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
    /* A layout's length is that of its parent_indices (QueryLayout.__len__,
     * runtime/execution/interfaces.py:96-97); reading the tuple directly
     * avoids one Python-level call per request. */
    Py_ssize_t len;
    int l = 1;
    if (!layout_shape(litems[r], &len, linear ? &l : NULL)) goto fail;
    if (len > INT32_MAX) {
      PyErr_SetString(PyExc_OverflowError, "step metadata count does not fit int32");
      goto fail;
    }
    qlen[r] = (int32_t)len;
    num_tokens += len;
    single += len == 1;
    if (len > max_query) max_query = len;
    if ((long long)comp[r] + len > max_seq) max_seq = (long long)comp[r] + len;
    linear = linear && l;
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

/* ------------------------------------------------------------------------
 * Call trampolines.  The attention step's library calls (lvb_paged_kv_write,
 * lvb_paged_attention) and the metadata staging call (lvb_stage_step_metadata)
 * take 17-30 arguments; through ctypes each call costs several microseconds of
 * argument conversion per layer and step.  bind() receives the three function
 * addresses once (from the ctypes library object); the entry points below
 * parse their arguments with the C API and call them directly.
 * ------------------------------------------------------------------------ */
typedef int (*kv_write_fn)(const void *, int64_t, const void *, int64_t, void *, void *, const void *, int64_t,
                           const void *, const void *, const void *, int64_t, int64_t, int64_t, int64_t, int,
                           void *);
typedef int (*attention_fn)(const void *, int64_t, const void *, const void *, void *, int64_t, const void *,
                            int64_t, const void *, const void *, const void *, const void *, const void *,
                            const void *, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                            int64_t, int64_t, float, int, void *, size_t, void *);
typedef int (*attention_kv_fn)(const void *, int64_t, const void *, int64_t, const void *, int64_t, void *, void *,
                               void *, int64_t, const void *, int64_t, const void *, const void *, const void *,
                               const void *, const void *, const void *, int64_t, int64_t, int64_t, int64_t,
                               int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float, int, void *, size_t,
                               void *);
typedef int (*stage_fn)(const int32_t *, const int64_t *, const int32_t *, const int32_t *, const int32_t *,
                        const int32_t *, int64_t, int64_t, int64_t, int32_t *, int64_t, int32_t *, int64_t, void *,
                        void *, int64_t *, int64_t *);
static kv_write_fn g_kv_write;
static attention_fn g_attention;
static stage_fn g_stage;
static attention_kv_fn g_attention_kv;

static PyObject *bind(PyObject *self, PyObject *args) {
  (void)self;
  unsigned long long kv, attn, stage, attn_kv;
  if (!PyArg_ParseTuple(args, "KKKK", &kv, &attn, &stage, &attn_kv)) return NULL;
  g_kv_write = (kv_write_fn)(uintptr_t)kv;
  g_attention = (attention_fn)(uintptr_t)attn;
  g_stage = (stage_fn)(uintptr_t)stage;
  g_attention_kv = (attention_kv_fn)(uintptr_t)attn_kv;
  Py_RETURN_NONE;
}

#define PTR(x) ((void *)(uintptr_t)(x))

/* attention_step(step, layer, q, q_stride, k, k_stride, v, v_stride, out,
 *                o_stride, write_kv, scale, workspace, workspace_bytes, stream)
 *   step  = (tables, table_stride, computed, query_start, request_indices,
 *            request_order, visibility, visibility_start, num_seqs,
 *            num_decode_seqs, num_tokens, max_query_len, max_seq_len)
 *   layer = (key_cache, value_cache, num_q_heads, num_kv_heads, head_size,
 *            block_size, num_blocks, dtype)
 * Runs lvb_paged_attention_kv (when write_kv: the step's K/V write and the
 * attention) or lvb_paged_attention; returns (status, 1) on failure.  The
 * failed_call value 0 (the K/V write) is kept for callers that name it. */
static PyObject *attention_step(PyObject *self, PyObject *args) {
  (void)self;
  unsigned long long tables, computed, qsl, req, order, vis, vis_start;
  long long stride, n_seqs, n_decode, n_tokens, max_q, max_seq;
  unsigned long long kc, vc;
  long long hq, hkv, d, bs, num_blocks;
  int dtype;
  unsigned long long q, k, v, out, ws, stream;
  long long q_stride, k_stride, v_stride, o_stride;
  int write_kv;
  float scale;
  Py_ssize_t ws_bytes;
  if (!PyArg_ParseTuple(args, "(KLKKKKKKLLLLL)(KKLLLLLi)KLKLKLKLpfKnK", &tables, &stride, &computed, &qsl, &req,
                        &order, &vis, &vis_start, &n_seqs, &n_decode, &n_tokens, &max_q, &max_seq, &kc, &vc, &hq,
                        &hkv, &d, &bs, &num_blocks, &dtype, &q, &q_stride, &k, &k_stride, &v, &v_stride, &out,
                        &o_stride, &write_kv, &scale, &ws, &ws_bytes, &stream))
    return NULL;
  if (!g_kv_write || !g_attention || !g_attention_kv) {
    PyErr_SetString(PyExc_RuntimeError, "_hostpack.bind was not called");
    return NULL;
  }
  if (write_kv) {
    /* One call: the decode path stores the step's rows itself. */
    const int rc = g_attention_kv(PTR(k), k_stride, PTR(v), v_stride, PTR(q), q_stride, PTR(kc), PTR(vc), PTR(out),
                                  o_stride, PTR(tables), stride, PTR(computed), PTR(qsl), PTR(req), PTR(order),
                                  PTR(vis), PTR(vis_start), n_seqs, n_decode, n_tokens, max_q, max_seq, hq, hkv, d,
                                  bs, num_blocks, scale, dtype, PTR(ws), (size_t)ws_bytes, PTR(stream));
    return Py_BuildValue("(ii)", rc, 1);
  }
  const int rc = g_attention(PTR(q), q_stride, PTR(kc), PTR(vc), PTR(out), o_stride, PTR(tables), stride,
                             PTR(computed), PTR(qsl), PTR(req), PTR(order), PTR(vis), PTR(vis_start), n_seqs,
                             n_decode, n_tokens, max_q, max_seq, hq, hkv, d, bs, num_blocks, scale, dtype, PTR(ws),
                             (size_t)ws_bytes, PTR(stream));
  return Py_BuildValue("(ii)", rc, 1);
}

/* stage_step(ids, offsets, rows, num_seqs, num_blocks, block_size, pinned,
 *            pinned_capacity, device, device_capacity, event, stream)
 *   -> (status, table_stride, num_tokens): lvb_stage_step_metadata over the
 *   buffers gather_step filled. */
static PyObject *stage_step(PyObject *self, PyObject *args) {
  (void)self;
  unsigned long long ids, offsets, rows, pinned, device, event, stream;
  long long n, num_blocks, block_size, pinned_cap, device_cap;
  if (!PyArg_ParseTuple(args, "KKKLLLKLKLKK", &ids, &offsets, &rows, &n, &num_blocks, &block_size, &pinned,
                        &pinned_cap, &device, &device_cap, &event, &stream))
    return NULL;
  if (!g_stage) {
    PyErr_SetString(PyExc_RuntimeError, "_hostpack.bind was not called");
    return NULL;
  }
  const int32_t *r = (const int32_t *)PTR(rows);
  int64_t stride = 0, ntok = 0;
  const int rc = g_stage((const int32_t *)PTR(ids), (const int64_t *)PTR(offsets), r, r + n, r + 2 * n, r + 3 * n, n,
                         num_blocks, block_size, (int32_t *)PTR(pinned), pinned_cap, (int32_t *)PTR(device),
                         device_cap, PTR(event), PTR(stream), &stride, &ntok);
  return Py_BuildValue("(iLL)", rc, (long long)stride, (long long)ntok);
}

static PyMethodDef methods[] = {
    {"bind", bind, METH_VARARGS,
     "bind(kv_write_addr, attention_addr, stage_addr, attention_kv_addr): library entry points"},
    {"attention_step", attention_step, METH_VARARGS,
     "attention_step(step, layer, q, q_stride, k, k_stride, v, v_stride, out, o_stride, write_kv, scale, "
     "workspace, workspace_bytes, stream) -> (status, failed_call)"},
    {"stage_step", stage_step, METH_VARARGS,
     "stage_step(ids, offsets, rows, n, num_blocks, block_size, pinned, pinned_capacity, device, "
     "device_capacity, event, stream) -> (status, table_stride, num_tokens)"},
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
