// _packnative: the per-sample half of packing runner trial records into the
// pm_trials structure of arrays, in C++ over the CPython object API.
//
// For every (trial, phase) slot it applies the reference's sample rules, as
// powermodeling_b200/pack.py states them in Python:
//  * _samples (powermodeling/analysis.py:85-91): items that are dicts with a
//    finite t_s, the last one of a repeated timestamp kept, ascending time;
//  * _finite (analysis.py:70-77) for every telemetry field: bools and values
//    float() rejects with TypeError/ValueError are None (NaN here), non-finite
//    values are None, float()'s other errors (an int too large) propagate;
//  * the energy counter kinds (anchor: exact int; nonnegative int or float),
//    the uint64 two's-complement fold of integer counters, _throttle_mask
//    (analysis.py:219-225; int(value, 0) for strings), the process-inventory
//    flags against the measurement pid, MPS, memory-power presence and the
//    memory-power source id table shared with the caller.
// It returns the columns as bytes (native byte order, pm_trials types), the
// sorted sample dicts of each slot and each slot's foreign pids, so the rest
// of the host code sees exactly what the Python packer produced.
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>

#include "pmb200.h"

namespace {

enum Key { K_T, K_POWER, K_MEMORY, K_GFX, K_SM, K_MEM, K_TEMP, K_PLIMIT, K_ENF, K_PSTATE, K_ENERGY, K_THROTTLE,
           K_COMPUTE, K_GRAPHICS, K_PID, K_MPS, K_SOURCE, K_COUNT };
const char* kKeyNames[K_COUNT] = {"t_s", "power_w", "memory_power_w", "graphics_clock_mhz", "sm_clock_mhz",
                                  "memory_clock_mhz", "temperature_c", "power_limit_w", "enforced_power_limit_w",
                                  "pstate", "energy_mj", "throttle_reasons", "compute_processes", "graphics_processes",
                                  "pid", "mps_compute_processes", "memory_power_source"};
PyObject* g_keys[K_COUNT];
PyObject* g_zero;       // int 0
PyObject* g_two64;      // int 2**64
const double kNaN = std::numeric_limits<double>::quiet_NaN();

// dict.get(key) as a borrowed reference (NULL: absent); -1 on error.
int get(PyObject* d, Key k, PyObject** out) {
  *out = PyDict_GetItemWithError(d, g_keys[k]);
  return (!*out && PyErr_Occurred()) ? -1 : 0;
}

// _finite: 1 and *out when finite, 0 for None, -1 with an exception set.
int finite(PyObject* v, double* out) {
  if (!v || v == Py_None || PyBool_Check(v)) return 0;
  double d;
  if (PyFloat_CheckExact(v)) {
    d = PyFloat_AS_DOUBLE(v);
  } else {
    PyObject* f = PyNumber_Float(v);
    if (!f) {
      if (PyErr_ExceptionMatches(PyExc_TypeError) || PyErr_ExceptionMatches(PyExc_ValueError)) {
        PyErr_Clear();
        return 0;
      }
      return -1;
    }
    d = PyFloat_AS_DOUBLE(f);
    Py_DECREF(f);
  }
  if (!std::isfinite(d)) return 0;
  *out = d;
  return 1;
}

int nan_if_none(PyObject* d, Key k, double* out) {
  PyObject* v;
  if (get(d, k, &v) < 0) return -1;
  double x;
  const int r = finite(v, &x);
  if (r < 0) return -1;
  *out = r ? x : kNaN;
  return 0;
}

// A Python int as the int64 the column stores: a value of 2**63 or more has
// 2**64 subtracted once (the uint64 counter's two's complement), a value below
// -2**63 becomes 0, and what still does not fit raises OverflowError, as
// numpy raises for it.
int fold_counter(PyObject* i, int64_t* out) {
  int overflow = 0;
  const long long v = PyLong_AsLongLongAndOverflow(i, &overflow);
  if (v == -1 && PyErr_Occurred()) return -1;
  if (overflow == 0) { *out = v; return 0; }
  if (overflow < 0) { *out = 0; return 0; }
  PyObject* folded = PyNumber_Subtract(i, g_two64);
  if (!folded) return -1;
  const long long f = PyLong_AsLongLong(folded);
  Py_DECREF(folded);
  if (f == -1 && PyErr_Occurred()) return -1;
  *out = f;
  return 0;
}

// _throttle_mask + the column's range rule: 1 and *out when the mask is in
// [-2**63, 2**64), 0 otherwise, -1 with an exception set.
int throttle(PyObject* v, int64_t* out) {
  if (!v || v == Py_None) return 0;
  PyObject* m = PyUnicode_Check(v) ? PyLong_FromUnicodeObject(v, 0) : PyNumber_Long(v);
  if (!m) {
    if (PyErr_ExceptionMatches(PyExc_TypeError) || PyErr_ExceptionMatches(PyExc_ValueError)) {
      PyErr_Clear();
      return 0;
    }
    return -1;
  }
  int overflow = 0;
  const long long s = PyLong_AsLongLongAndOverflow(m, &overflow);
  int result = 0;
  if (s == -1 && PyErr_Occurred()) {
    result = -1;
  } else if (overflow == 0) {
    *out = s;
    result = 1;
  } else if (overflow > 0) {
    const unsigned long long u = PyLong_AsUnsignedLongLong(m);
    if (u == (unsigned long long)-1 && PyErr_Occurred()) {
      if (PyErr_ExceptionMatches(PyExc_OverflowError)) { PyErr_Clear(); result = 0; }
      else result = -1;
    } else {
      *out = (int64_t)u;
      result = 1;
    }
  }
  Py_DECREF(m);
  return result;
}

struct Columns {
  std::vector<double> t, power, memory, gfx, sm, mem, temp, plimit, enf, pstate, e_float;
  std::vector<int64_t> e_int, throttle;
  std::vector<uint16_t> flags;
  std::vector<uint8_t> source;
};

// Source ids: 0 for a false value, else 1 + (table size when first seen) mod 15,
// keyed by the string or its repr; `table` is the caller's dict.
int source_id(PyObject* source, PyObject* table, uint8_t* out) {
  *out = 0;
  if (!source) return 0;
  const int truth = PyObject_IsTrue(source);
  if (truth < 0) return -1;
  if (!truth) return 0;
  PyObject* key = PyUnicode_Check(source) ? (Py_INCREF(source), source) : PyObject_Repr(source);
  if (!key) return -1;
  PyObject* id = PyDict_GetItemWithError(table, key);
  if (!id) {
    if (PyErr_Occurred()) { Py_DECREF(key); return -1; }
    PyObject* fresh = PyLong_FromSsize_t(1 + PyDict_Size(table) % 15);
    if (!fresh || PyDict_SetItem(table, key, fresh) < 0) { Py_XDECREF(fresh); Py_DECREF(key); return -1; }
    Py_DECREF(fresh);
    id = PyDict_GetItemWithError(table, key);
  }
  Py_DECREF(key);
  if (!id) return -1;
  const long v = PyLong_AsLong(id);
  if (v == -1 && PyErr_Occurred()) return -1;
  *out = (uint8_t)v;
  return 0;
}

// One sample dict into the columns; foreign pids appended to `foreign`.
int pack_sample(PyObject* s, PyObject* pid, PyObject* table, Columns& c, PyObject* foreign) {
  PyObject* v;
  if (get(s, K_T, &v) < 0) return -1;
  if (!v) { PyErr_SetObject(PyExc_KeyError, g_keys[K_T]); return -1; }
  double t;
  if (PyFloat_CheckExact(v)) {
    t = PyFloat_AS_DOUBLE(v);
  } else {                                  // float(s["t_s"]): strings parse as float() parses them
    PyObject* f = PyNumber_Float(v);
    if (!f) return -1;
    t = PyFloat_AS_DOUBLE(f);
    Py_DECREF(f);
  }
  c.t.push_back(t);
  double x;
  const Key fields[9] = {K_POWER, K_MEMORY, K_GFX, K_SM, K_MEM, K_TEMP, K_PLIMIT, K_ENF, K_PSTATE};
  std::vector<double>* cols[9] = {&c.power, &c.memory, &c.gfx, &c.sm, &c.mem, &c.temp, &c.plimit, &c.enf, &c.pstate};
  for (int k = 0; k < 9; ++k) {
    if (nan_if_none(s, fields[k], &x) < 0) return -1;
    cols[k]->push_back(x);
  }
  uint32_t flags = 0;
  int64_t e_int = 0;
  double e_float = kNaN;
  PyObject* counter;
  if (get(s, K_ENERGY, &counter) < 0) return -1;
  if (counter) {
    if (PyLong_CheckExact(counter)) {
      flags |= PM_S_ENERGY_ANCHOR;
      if (fold_counter(counter, &e_int) < 0) return -1;
    }
    if ((PyLong_Check(counter) || PyFloat_Check(counter)) && !PyBool_Check(counter)) {
      const int nonneg = PyObject_RichCompareBool(counter, g_zero, Py_GE);
      if (nonneg < 0) return -1;
      if (nonneg) {
        if (PyLong_Check(counter)) {
          flags |= PM_S_ENERGY_INT;
          if (fold_counter(counter, &e_int) < 0) return -1;
        } else {
          flags |= PM_S_ENERGY_FLOAT;
          e_float = PyFloat_AsDouble(counter);
          if (e_float == -1.0 && PyErr_Occurred()) return -1;
        }
      }
    }
  }
  c.e_int.push_back(e_int);
  c.e_float.push_back(e_float);
  PyObject* tr;
  if (get(s, K_THROTTLE, &tr) < 0) return -1;
  int64_t mask = 0;
  const int tm = throttle(tr, &mask);
  if (tm < 0) return -1;
  if (tm) flags |= PM_S_THROTTLE_VALID;
  c.throttle.push_back(tm ? mask : 0);
  const Key inventories[2] = {K_COMPUTE, K_GRAPHICS};
  const uint32_t missing[2] = {PM_S_NO_COMPUTE_INV, PM_S_NO_GRAPHICS_INV};
  for (int j = 0; j < 2; ++j) {
    PyObject* inv;
    if (get(s, inventories[j], &inv) < 0) return -1;
    if (!inv || !PyList_Check(inv)) { flags |= missing[j]; continue; }
    if (PyList_GET_SIZE(inv) > 0 && pid == Py_None) flags |= PM_S_PID_UNKNOWN;
    for (Py_ssize_t q = 0; q < PyList_GET_SIZE(inv); ++q) {
      PyObject* process = PyList_GET_ITEM(inv, q);
      PyObject* p = process;
      if (PyDict_Check(process)) {
        if (get(process, K_PID, &p) < 0) return -1;
        if (!p) p = Py_None;
      }
      Py_INCREF(p);
      const int ne = PyObject_RichCompareBool(p, pid, Py_NE);
      if (ne < 0) { Py_DECREF(p); return -1; }
      if (ne) flags |= PM_S_REF_FOREIGN;
      if (ne && p != Py_None) {
        flags |= PM_S_FOREIGN_PID;
        if (PyList_Append(foreign, p) < 0) { Py_DECREF(p); return -1; }
      }
      Py_DECREF(p);
    }
  }
  PyObject* mps;
  if (get(s, K_MPS, &mps) < 0) return -1;
  if (mps) {
    const int truth = PyObject_IsTrue(mps);
    if (truth < 0) return -1;
    if (truth) flags |= PM_S_MPS;
  }
  PyObject* mp;
  if (get(s, K_MEMORY, &mp) < 0) return -1;
  if (mp && mp != Py_None) flags |= PM_S_MEMORY_POWER_SET;
  PyObject* src;
  if (get(s, K_SOURCE, &src) < 0) return -1;
  uint8_t sid = 0;
  if (source_id(src, table, &sid) < 0) return -1;
  c.source.push_back(sid);
  c.flags.push_back((uint16_t)flags);
  return 0;
}

// _samples over one slot's raw samples: a new list of the kept dicts in time order.
PyObject* sorted_samples(PyObject* raw) {
  struct Item { double t; Py_ssize_t index; PyObject* item; };
  std::vector<Item> items;
  PyObject* it = PyObject_GetIter(raw);
  if (!it) return nullptr;
  Py_ssize_t index = 0;
  PyObject* holder = PyList_New(0);   // keeps every candidate alive while sorting
  if (!holder) { Py_DECREF(it); return nullptr; }
  while (PyObject* item = PyIter_Next(it)) {
    if (PyList_Append(holder, item) < 0) { Py_DECREF(item); Py_DECREF(it); Py_DECREF(holder); return nullptr; }
    Py_DECREF(item);
    if (!PyDict_Check(item)) { ++index; continue; }
    PyObject* tv;
    if (get(item, K_T, &tv) < 0) { Py_DECREF(it); Py_DECREF(holder); return nullptr; }
    double t;
    const int r = finite(tv, &t);
    if (r < 0) { Py_DECREF(it); Py_DECREF(holder); return nullptr; }
    if (r) items.push_back({t, index, item});
    ++index;
  }
  Py_DECREF(it);
  if (PyErr_Occurred()) { Py_DECREF(holder); return nullptr; }
  std::stable_sort(items.begin(), items.end(), [](const Item& a, const Item& b) { return a.t < b.t; });
  PyObject* out = PyList_New(0);
  if (!out) { Py_DECREF(holder); return nullptr; }
  for (size_t k = 0; k < items.size(); ++k) {
    // Equal timestamps (0.0 == -0.0 included) form one dict key: the last item wins.
    if (k + 1 < items.size() && items[k + 1].t == items[k].t) continue;
    if (PyList_Append(out, items[k].item) < 0) { Py_DECREF(out); Py_DECREF(holder); return nullptr; }
  }
  Py_DECREF(holder);
  return out;
}

template <class T>
PyObject* as_bytes(const std::vector<T>& v) {
  return PyBytes_FromStringAndSize(reinterpret_cast<const char*>(v.data()), (Py_ssize_t)(v.size() * sizeof(T)));
}

// pack(slots, pids, source_ids) -> (columns, counts, sorted, foreign)
//   slots: list of iterables of raw samples (one per (trial, phase) slot)
//   pids: list of the measurement pid of each slot's trial
//   source_ids: dict shared with the caller (memory-power source -> id)
PyObject* pack(PyObject*, PyObject* args) {
  PyObject *slots, *pids, *table;
  if (!PyArg_ParseTuple(args, "O!O!O!", &PyList_Type, &slots, &PyList_Type, &pids, &PyDict_Type, &table)) return nullptr;
  const Py_ssize_t n = PyList_GET_SIZE(slots);
  if (PyList_GET_SIZE(pids) != n) { PyErr_SetString(PyExc_ValueError, "slots and pids differ in length"); return nullptr; }
  Columns c;
  PyObject* counts = PyList_New(n);
  PyObject* sorted = PyList_New(n);
  PyObject* foreign = PyList_New(n);
  if (!counts || !sorted || !foreign) { Py_XDECREF(counts); Py_XDECREF(sorted); Py_XDECREF(foreign); return nullptr; }
  auto fail = [&]() -> PyObject* { Py_DECREF(counts); Py_DECREF(sorted); Py_DECREF(foreign); return nullptr; };
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* samples = sorted_samples(PyList_GET_ITEM(slots, i));
    if (!samples) return fail();
    PyList_SET_ITEM(sorted, i, samples);
    PyObject* slot_foreign = PyList_New(0);
    if (!slot_foreign) return fail();
    PyList_SET_ITEM(foreign, i, slot_foreign);
    PyObject* pid = PyList_GET_ITEM(pids, i);
    const Py_ssize_t m = PyList_GET_SIZE(samples);
    for (Py_ssize_t k = 0; k < m; ++k) {
      PyObject* found = PyList_New(0);
      if (!found) return fail();
      if (pack_sample(PyList_GET_ITEM(samples, k), pid, table, c, found) < 0) { Py_DECREF(found); return fail(); }
      if (PyList_GET_SIZE(found) > 0) {
        PyObject* entry = Py_BuildValue("(nN)", k, found);
        if (!entry || PyList_Append(slot_foreign, entry) < 0) { Py_XDECREF(entry); return fail(); }
        Py_DECREF(entry);
      } else {
        Py_DECREF(found);
      }
    }
    PyObject* count = PyLong_FromSsize_t(m);
    if (!count) return fail();
    PyList_SET_ITEM(counts, i, count);
  }
  PyObject* columns = Py_BuildValue("{s:N,s:N,s:N,s:N,s:N,s:N,s:N,s:N,s:N,s:N,s:N,s:N,s:N,s:N,s:N}",
      "t_s", as_bytes(c.t), "power_w", as_bytes(c.power), "memory_power_w", as_bytes(c.memory),
      "graphics_clock_mhz", as_bytes(c.gfx), "sm_clock_mhz", as_bytes(c.sm), "memory_clock_mhz", as_bytes(c.mem),
      "temperature_c", as_bytes(c.temp), "power_limit_w", as_bytes(c.plimit),
      "enforced_power_limit_w", as_bytes(c.enf), "pstate", as_bytes(c.pstate), "energy_int", as_bytes(c.e_int),
      "energy_float", as_bytes(c.e_float), "throttle_reasons", as_bytes(c.throttle),
      "sample_flags", as_bytes(c.flags), "memory_power_source", as_bytes(c.source));
  if (!columns) return fail();
  return Py_BuildValue("(NNNN)", columns, counts, sorted, foreign);
}

PyMethodDef kMethods[] = {
    {"pack", pack, METH_VARARGS, "pack(slots, pids, source_ids) -> (columns, counts, sorted, foreign)"},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_packnative",
                       "Per-sample packing of runner trial records into pm_trials columns.", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__packnative(void) {
  for (int k = 0; k < K_COUNT; ++k) {
    g_keys[k] = PyUnicode_InternFromString(kKeyNames[k]);
    if (!g_keys[k]) return nullptr;
  }
  g_zero = PyLong_FromLong(0);
  PyObject* one = PyLong_FromLong(1), *sixty_four = PyLong_FromLong(64);
  g_two64 = one && sixty_four ? PyNumber_Lshift(one, sixty_four) : nullptr;
  Py_XDECREF(one);
  Py_XDECREF(sixty_four);
  if (!g_zero || !g_two64) return nullptr;
  return PyModule_Create(&kModule);
}
