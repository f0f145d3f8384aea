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
#include <sched.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <thread>
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

// ---------------------------------------------------------------------------
// Parallel fast path.
//
// Most records hold plain data: lists of exact dicts whose values are exact
// floats, small exact ints, None, bools and empty or small lists.  For those,
// worker threads read the dicts directly while the calling thread holds the
// GIL and waits for them, so no Python code can run, allocate, free or mutate
// anything meanwhile.  The workers only read immutable payloads (float
// values, compact int digits, string bytes) and dict and list entry tables;
// they never change a reference count, allocate a Python object or raise.
// A slot holding anything else (strings to parse, big ints, subclasses,
// objects with __float__, unusual process entries) is marked and packed by
// the object-API path above on the calling thread, so both paths produce
// exactly what the Python packer specifies.
//
// Pass one reads every sample dict of a slot once (its values under our
// keys), keeps the samples with a finite time in time order and counts them;
// the calling thread then places every slot in the output columns; pass two
// converts the kept samples straight into the final column buffers.
struct SlotPlan {
  bool fast = false;                   // packed by the workers
  Py_ssize_t base = 0;                 // first output row
  std::vector<Py_ssize_t> order;       // kept items of the raw list, in time order
  std::vector<double> t;               // their times
  std::vector<PyObject*> vals;         // per raw item, its values under our keys (borrowed, NULL: absent)
  std::vector<uint8_t> source_ids;     // per kept sample, numbered on the calling thread in slot order
  std::vector<std::pair<Py_ssize_t, std::vector<PyObject*>>> foreign;   // (kept position, borrowed pids)
};

// Output columns in their final buffers (bytes objects the calling thread allocated).
struct OutColumns {
  double *t, *power, *memory, *gfx, *sm, *mem, *temp, *plimit, *enf, *pstate, *e_float;
  int64_t *e_int, *throttle;
  uint16_t* flags;
  uint8_t* source;
  uint8_t* clock_repeat;   // host only: 1 when a sample's clocks repeat the previous kept sample's
};



// Key of an exact str by content (-1: not one of ours, -2: not an exact str), with a pointer cache per worker.
struct KeyCache {
  PyObject* key[64] = {};
  int8_t index[64] = {};
  size_t length[K_COUNT];
  KeyCache() { for (int j = 0; j < K_COUNT; ++j) length[j] = strlen(kKeyNames[j]); }
  int find(PyObject* k) {
    const size_t h = (reinterpret_cast<uintptr_t>(k) >> 4) & 63;
    if (key[h] == k) return index[h];
    int found = -1;
    if (!PyUnicode_CheckExact(k)) {
      found = -2;                      // equality of such a key with our names is the object API's call
    } else if (PyUnicode_KIND(k) == PyUnicode_1BYTE_KIND) {
      const size_t n = (size_t)PyUnicode_GET_LENGTH(k);
      const char* data = reinterpret_cast<const char*>(PyUnicode_1BYTE_DATA(k));
      for (int j = 0; j < K_COUNT; ++j)
        if (length[j] == n && memcmp(kKeyNames[j], data, n) == 0) { found = j; break; }
    }
    key[h] = k;
    index[h] = (int8_t)found;
    return found;
  }
};

bool compact_int(PyObject* v, int64_t* out) {
  if (!PyLong_CheckExact(v) || !PyUnstable_Long_IsCompact(reinterpret_cast<PyLongObject*>(v))) return false;
  *out = (int64_t)PyUnstable_Long_CompactValue(reinterpret_cast<PyLongObject*>(v));
  return true;
}

// Two telemetry values that read back as the same Python value: the same object, None and an
// absent key, exact floats with the same bits, or exact compact ints of the same value.
bool same_value(PyObject* a, PyObject* b) {
  if (!a) a = Py_None;
  if (!b) b = Py_None;
  if (a == b) return true;
  if (PyFloat_CheckExact(a) && PyFloat_CheckExact(b)) {
    const double x = PyFloat_AS_DOUBLE(a), y = PyFloat_AS_DOUBLE(b);
    return memcmp(&x, &y, sizeof x) == 0;
  }
  int64_t i, j;
  return compact_int(a, &i) && compact_int(b, &j) && i == j;
}

// _finite on plain values: 1 finite (*out), 0 None/absent/bool/non-finite, -1 needs the object API.
int plain_finite(PyObject* v, double* out) {
  if (!v || v == Py_None || PyBool_Check(v)) return 0;
  if (PyFloat_CheckExact(v)) {
    const double d = PyFloat_AS_DOUBLE(v);
    if (!std::isfinite(d)) return 0;
    *out = d;
    return 1;
  }
  int64_t i;
  if (compact_int(v, &i)) { *out = (double)i; return 1; }
  return -1;
}

// The dict's values under our keys (NULL: absent); false when a key needs the object API.
bool read_keys(PyObject* d, KeyCache& cache, PyObject** vals) {
  for (int j = 0; j < K_COUNT; ++j) vals[j] = nullptr;
  Py_ssize_t pos = 0;
  PyObject *k, *v;
  while (PyDict_Next(d, &pos, &k, &v)) {
    const int j = cache.find(k);
    if (j == -2) return false;
    if (j >= 0) vals[j] = v;
  }
  return true;
}

// Inventory entry pid against the measurement pid: 1 differs, 0 equal, -1 needs the object API.
int plain_differs(PyObject* p, PyObject* pid) {
  if (p == pid) return 0;
  if (p == Py_None || pid == Py_None) return 1;
  int64_t a, b;
  if (compact_int(p, &a) && compact_int(pid, &b)) return a != b;
  return -1;
}

// Pass one: read, keep and order a slot's samples.
bool plan_slot(PyObject* raw, SlotPlan& plan, KeyCache& cache) {
  const Py_ssize_t n = PyList_GET_SIZE(raw);
  struct Item { double t; Py_ssize_t index; };
  std::vector<Item> items;
  items.reserve((size_t)n);
  plan.vals.assign((size_t)n * K_COUNT, nullptr);
  bool ascending = true;
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* item = PyList_GET_ITEM(raw, i);
    if (!PyDict_Check(item)) continue;            // not a sample (the reference skips it)
    if (!PyDict_CheckExact(item)) return false;
    PyObject** v = &plan.vals[(size_t)i * K_COUNT];
    if (!read_keys(item, cache, v)) return false;
    double t;
    const int r = plain_finite(v[K_T], &t);
    if (r < 0) return false;
    if (!r) continue;
    if (!items.empty() && !(items.back().t < t)) ascending = false;
    items.push_back({t, i});
  }
  if (!ascending) {
    std::stable_sort(items.begin(), items.end(), [](const Item& a, const Item& b) { return a.t < b.t; });
    size_t w = 0;
    for (size_t k = 0; k < items.size(); ++k)     // equal timestamps: the last one wins
      if (!(k + 1 < items.size() && items[k + 1].t == items[k].t)) items[w++] = items[k];
    items.resize(w);
  }
  plan.order.resize(items.size());
  plan.t.resize(items.size());
  for (size_t k = 0; k < items.size(); ++k) { plan.order[k] = items[k].index; plan.t[k] = items[k].t; }
  return true;
}

// Pass two: the kept samples into rows base.. of the output.
bool fill_slot(SlotPlan& plan, PyObject* pid, KeyCache& cache, const OutColumns& c) {
  const Key fields[9] = {K_POWER, K_MEMORY, K_GFX, K_SM, K_MEM, K_TEMP, K_PLIMIT, K_ENF, K_PSTATE};
  double* cols[9] = {c.power, c.memory, c.gfx, c.sm, c.mem, c.temp, c.plimit, c.enf, c.pstate};
  std::vector<PyObject*> found;
  const size_t m = plan.order.size();
  for (size_t k = 0; k < m; ++k) {
    const size_t row = (size_t)plan.base + k;
    PyObject** v = &plan.vals[(size_t)plan.order[k] * K_COUNT];
    c.t[row] = plan.t[k];
    if (k == 0) {
      c.clock_repeat[row] = 0;
    } else {
      PyObject** u = &plan.vals[(size_t)plan.order[k - 1] * K_COUNT];
      c.clock_repeat[row] = same_value(v[K_GFX], u[K_GFX]) && same_value(v[K_MEM], u[K_MEM]) ? 1 : 0;
    }
    for (int j = 0; j < 9; ++j) {
      double x;
      const int r = plain_finite(v[fields[j]], &x);
      if (r < 0) return false;
      cols[j][row] = r ? x : kNaN;
    }
    uint32_t flags = 0;
    int64_t e_int = 0;
    double e_float = kNaN;
    if (PyObject* e = v[K_ENERGY]; e && e != Py_None && !PyBool_Check(e)) {
      int64_t i;
      if (compact_int(e, &i)) {
        flags |= PM_S_ENERGY_ANCHOR;
        e_int = i;
        if (i >= 0) flags |= PM_S_ENERGY_INT;
      } else if (PyFloat_CheckExact(e)) {
        if (PyFloat_AS_DOUBLE(e) >= 0) { flags |= PM_S_ENERGY_FLOAT; e_float = PyFloat_AS_DOUBLE(e); }
      } else {
        return false;
      }
    }
    c.e_int[row] = e_int;
    c.e_float[row] = e_float;
    int64_t mask = 0;
    if (PyObject* tr = v[K_THROTTLE]; tr && tr != Py_None) {
      if (!compact_int(tr, &mask)) return false;
      flags |= PM_S_THROTTLE_VALID;
    }
    c.throttle[row] = mask;
    const Key inventories[2] = {K_COMPUTE, K_GRAPHICS};
    const uint32_t missing[2] = {PM_S_NO_COMPUTE_INV, PM_S_NO_GRAPHICS_INV};
    found.clear();
    for (int j = 0; j < 2; ++j) {
      PyObject* inv = v[inventories[j]];
      if (!inv || !PyList_Check(inv)) { flags |= missing[j]; continue; }
      if (!PyList_CheckExact(inv)) return false;
      const Py_ssize_t q = PyList_GET_SIZE(inv);
      if (q > 0 && pid == Py_None) flags |= PM_S_PID_UNKNOWN;
      for (Py_ssize_t e = 0; e < q; ++e) {
        PyObject* entry = PyList_GET_ITEM(inv, e);
        PyObject* p = entry;
        if (PyDict_Check(entry)) {
          if (!PyDict_CheckExact(entry)) return false;
          PyObject* ev[K_COUNT];
          if (!read_keys(entry, cache, ev)) return false;
          p = ev[K_PID] ? ev[K_PID] : Py_None;
        }
        const int ne = plain_differs(p, pid);
        if (ne < 0) return false;
        if (ne) {
          flags |= PM_S_REF_FOREIGN;
          if (p != Py_None) { flags |= PM_S_FOREIGN_PID; found.push_back(p); }
        }
      }
    }
    if (!found.empty()) plan.foreign.emplace_back((Py_ssize_t)k, found);
    if (PyObject* mps = v[K_MPS]) {
      if (PyList_CheckExact(mps)) { if (PyList_GET_SIZE(mps) > 0) flags |= PM_S_MPS; }
      else if (mps == Py_True) flags |= PM_S_MPS;
      else if (mps != Py_None && mps != Py_False) return false;
    }
    if (v[K_MEMORY] && v[K_MEMORY] != Py_None) flags |= PM_S_MEMORY_POWER_SET;
    c.source[row] = plan.source_ids[k];
    c.flags[row] = (uint16_t)flags;
  }
  return true;
}

// Slots the last pack() call packed on the fast path (for tests and diagnostics).
Py_ssize_t g_last_fast_slots = 0;

// Worker threads: PM_PACK_THREADS, else the CPUs this process may run on (its
// affinity mask, which a launcher that pins one process per GPU narrows), at most 16: on a
// 16-CPU host the 64 x 4 sweep packs in 14.9 ms on 16 threads against 16.7 ms on 8 and
// 14.3 ms on 32, where the oversubscribed workers then slow the rest of the call.
int pack_threads() {
  static const int n = [] {
    const char* env = getenv("PM_PACK_THREADS");
    cpu_set_t set;
    int cpus = sched_getaffinity(0, sizeof(set), &set) == 0 ? CPU_COUNT(&set)
                                                           : (int)std::thread::hardware_concurrency();
    int v = env ? atoi(env) : std::min(16, std::max(1, cpus));
    return std::max(1, std::min(v, 64));
  }();
  return n;
}

// Runs fn(slot index) over `slots` on up to `workers` threads (the calling thread included).
template <class F>
void parallel_for(const std::vector<Py_ssize_t>& slots, int workers, F fn) {
  std::atomic<size_t> next{0};
  auto work = [&] {
    for (size_t j; (j = next.fetch_add(1)) < slots.size();) fn(slots[j]);
  };
  std::vector<std::thread> pool;
  for (int w = 1; w < workers; ++w) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
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
  std::vector<SlotPlan> plans((size_t)n);
  std::vector<Py_ssize_t> lists;
  Py_ssize_t raw_total = 0;
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* raw = PyList_GET_ITEM(slots, i);
    if (PyList_CheckExact(raw)) { lists.push_back(i); raw_total += PyList_GET_SIZE(raw); }
  }
  const int workers = raw_total >= 4096 ? std::min<int>(pack_threads(), (int)lists.size()) : 1;
  parallel_for(lists, workers, [&](Py_ssize_t i) {
    KeyCache cache;
    SlotPlan& plan = plans[(size_t)i];
    plan.fast = plan_slot(PyList_GET_ITEM(slots, i), plan, cache);
    if (!plan.fast) plan = SlotPlan{};
  });
  // Every other slot through the object-API path, then every slot's place in the output.
  std::vector<PyObject*> sorted_lists((size_t)n, nullptr);
  std::vector<Columns> slow((size_t)n);
  std::vector<PyObject*> slow_foreign((size_t)n, nullptr);
  auto release = [&] {
    for (PyObject* o : sorted_lists) Py_XDECREF(o);
    for (PyObject* o : slow_foreign) Py_XDECREF(o);
  };
  // Memory-power sources are numbered in first-seen order over slots and samples, so every
  // slot's sources are numbered here, in slot order, whichever path packs it.
  Py_ssize_t rows = 0;
  PyObject* cached_source = nullptr;
  uint8_t cached_id = 0;
  for (Py_ssize_t i = 0; i < n; ++i) {
    SlotPlan& plan = plans[(size_t)i];
    plan.base = rows;
    if (plan.fast) {
      plan.source_ids.resize(plan.order.size());
      for (size_t k = 0; k < plan.order.size(); ++k) {
        PyObject* src = plan.vals[(size_t)plan.order[k] * K_COUNT + K_SOURCE];
        if (src && src != cached_source) {
          if (source_id(src, table, &cached_id) < 0) { release(); return nullptr; }
          cached_source = src;
        }
        plan.source_ids[k] = src ? cached_id : 0;
      }
      rows += (Py_ssize_t)plan.order.size();
      continue;
    }
    cached_source = nullptr;
    PyObject* samples = sorted_samples(PyList_GET_ITEM(slots, i));
    if (!samples) { release(); return nullptr; }
    sorted_lists[(size_t)i] = samples;
    PyObject* slot_foreign = PyList_New(0);
    if (!slot_foreign) { release(); return nullptr; }
    slow_foreign[(size_t)i] = slot_foreign;
    const Py_ssize_t m = PyList_GET_SIZE(samples);
    for (Py_ssize_t k = 0; k < m; ++k) {
      PyObject* found = PyList_New(0);
      if (!found) { release(); return nullptr; }
      if (pack_sample(PyList_GET_ITEM(samples, k), PyList_GET_ITEM(pids, i), table, slow[(size_t)i], found) < 0) {
        Py_DECREF(found); release(); return nullptr;
      }
      if (PyList_GET_SIZE(found) > 0) {
        PyObject* entry = Py_BuildValue("(nN)", k, found);
        if (!entry || PyList_Append(slot_foreign, entry) < 0) { Py_XDECREF(entry); release(); return nullptr; }
        Py_DECREF(entry);
      } else {
        Py_DECREF(found);
      }
    }
    rows += m;
  }
  // The output columns, allocated once; pass two fills the fast slots' rows in parallel.
  const char* names[16] = {"t_s", "power_w", "memory_power_w", "graphics_clock_mhz", "sm_clock_mhz", "memory_clock_mhz",
                           "temperature_c", "power_limit_w", "enforced_power_limit_w", "pstate", "energy_int",
                           "energy_float", "throttle_reasons", "sample_flags", "memory_power_source", "clock_repeat"};
  const size_t widths[16] = {8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 8, 2, 1, 1};
  PyObject* columns = PyDict_New();
  if (!columns) { release(); return nullptr; }
  char* buf[16];
  for (int j = 0; j < 16; ++j) {
    PyObject* b = PyByteArray_FromStringAndSize(nullptr, (Py_ssize_t)(rows * widths[j]));
    if (!b || PyDict_SetItemString(columns, names[j], b) < 0) { Py_XDECREF(b); Py_DECREF(columns); release(); return nullptr; }
    Py_DECREF(b);
    buf[j] = PyByteArray_AS_STRING(b);
  }
  const OutColumns out{reinterpret_cast<double*>(buf[0]), reinterpret_cast<double*>(buf[1]),
                       reinterpret_cast<double*>(buf[2]), reinterpret_cast<double*>(buf[3]),
                       reinterpret_cast<double*>(buf[4]), reinterpret_cast<double*>(buf[5]),
                       reinterpret_cast<double*>(buf[6]), reinterpret_cast<double*>(buf[7]),
                       reinterpret_cast<double*>(buf[8]), reinterpret_cast<double*>(buf[9]),
                       reinterpret_cast<double*>(buf[11]), reinterpret_cast<int64_t*>(buf[10]),
                       reinterpret_cast<int64_t*>(buf[12]), reinterpret_cast<uint16_t*>(buf[13]),
                       reinterpret_cast<uint8_t*>(buf[14]), reinterpret_cast<uint8_t*>(buf[15])};
  std::vector<Py_ssize_t> fast;
  for (Py_ssize_t i = 0; i < n; ++i)
    if (plans[(size_t)i].fast) fast.push_back(i);
  std::vector<char> refill((size_t)n, 0);        // a fast slot pass two could not convert
  parallel_for(fast, workers, [&](Py_ssize_t i) {
    KeyCache cache;
    if (!fill_slot(plans[(size_t)i], PyList_GET_ITEM(pids, i), cache, out)) refill[(size_t)i] = 1;
  });
  // Slots pass two gave up on: the object-API path into the same rows.
  for (Py_ssize_t i : fast) {
    if (!refill[(size_t)i]) continue;
    SlotPlan& plan = plans[(size_t)i];
    plan.fast = false;
    PyObject* samples = sorted_samples(PyList_GET_ITEM(slots, i));
    PyObject* slot_foreign = samples ? PyList_New(0) : nullptr;
    if (!slot_foreign) { Py_XDECREF(samples); Py_DECREF(columns); release(); return nullptr; }
    sorted_lists[(size_t)i] = samples;
    slow_foreign[(size_t)i] = slot_foreign;
    for (Py_ssize_t k = 0; k < PyList_GET_SIZE(samples); ++k) {
      PyObject* found = PyList_New(0);
      if (!found || pack_sample(PyList_GET_ITEM(samples, k), PyList_GET_ITEM(pids, i), table, slow[(size_t)i], found) < 0) {
        Py_XDECREF(found); Py_DECREF(columns); release(); return nullptr;
      }
      if (PyList_GET_SIZE(found) > 0) {
        PyObject* entry = Py_BuildValue("(nN)", k, found);
        if (!entry || PyList_Append(slot_foreign, entry) < 0) { Py_XDECREF(entry); Py_DECREF(columns); release(); return nullptr; }
        Py_DECREF(entry);
      } else {
        Py_DECREF(found);
      }
    }
  }
  // Object-API slots: their columns into their rows.
  for (Py_ssize_t i = 0; i < n; ++i) {
    if (plans[(size_t)i].fast) continue;
    const Columns& c = slow[(size_t)i];
    const size_t b = (size_t)plans[(size_t)i].base, m = c.t.size();
    auto put = [&](auto* dst, const auto& src) { if (m) memcpy(dst + b, src.data(), m * sizeof(src[0])); };
    put(out.t, c.t); put(out.power, c.power); put(out.memory, c.memory); put(out.gfx, c.gfx); put(out.sm, c.sm);
    put(out.mem, c.mem); put(out.temp, c.temp); put(out.plimit, c.plimit); put(out.enf, c.enf);
    put(out.pstate, c.pstate); put(out.e_float, c.e_float); put(out.e_int, c.e_int); put(out.throttle, c.throttle);
    put(out.flags, c.flags); put(out.source, c.source);
    if (m) memset(out.clock_repeat + b, 0, m);    // these slots' bindings read every sample
  }
  g_last_fast_slots = (Py_ssize_t)std::count_if(plans.begin(), plans.end(), [](const SlotPlan& p) { return p.fast; });
  PyObject* counts = PyList_New(n);
  PyObject* sorted = PyList_New(n);
  PyObject* foreign = PyList_New(n);
  auto fail = [&]() -> PyObject* {
    Py_XDECREF(counts); Py_XDECREF(sorted); Py_XDECREF(foreign); Py_DECREF(columns); release(); return nullptr;
  };
  if (!counts || !sorted || !foreign) return fail();
  for (Py_ssize_t i = 0; i < n; ++i) {
    SlotPlan& plan = plans[(size_t)i];
    PyObject* raw = PyList_GET_ITEM(slots, i);
    Py_ssize_t m;
    if (!plan.fast) {
      PyList_SET_ITEM(sorted, i, sorted_lists[(size_t)i]);
      sorted_lists[(size_t)i] = nullptr;
      PyList_SET_ITEM(foreign, i, slow_foreign[(size_t)i]);
      slow_foreign[(size_t)i] = nullptr;
      m = PyList_GET_SIZE(PyList_GET_ITEM(sorted, i));
    } else {
      m = (Py_ssize_t)plan.order.size();
      // A raw list already in time order with every item kept is its own sorted
      // list (the packer never mutates it): no new list and no per-sample
      // reference count to touch (each sample dict is a cache miss).
      bool whole = m == PyList_GET_SIZE(raw);
      for (Py_ssize_t k = 0; whole && k < m; ++k) whole = plan.order[(size_t)k] == k;
      PyObject* samples = whole ? (Py_INCREF(raw), raw) : PyList_New(m);
      if (!samples) return fail();
      PyList_SET_ITEM(sorted, i, samples);
      for (Py_ssize_t k = 0; !whole && k < m; ++k) {
        PyObject* item = PyList_GET_ITEM(raw, plan.order[(size_t)k]);
        Py_INCREF(item);
        PyList_SET_ITEM(samples, k, item);
      }
      PyObject* slot_foreign = PyList_New(0);
      if (!slot_foreign) return fail();
      PyList_SET_ITEM(foreign, i, slot_foreign);
      for (auto& [k, found_pids] : plan.foreign) {
        PyObject* found = PyList_New((Py_ssize_t)found_pids.size());
        if (!found) return fail();
        for (size_t q = 0; q < found_pids.size(); ++q) {
          Py_INCREF(found_pids[q]);
          PyList_SET_ITEM(found, (Py_ssize_t)q, found_pids[q]);
        }
        PyObject* entry = Py_BuildValue("(nN)", k, found);
        if (!entry || PyList_Append(slot_foreign, entry) < 0) { Py_XDECREF(entry); return fail(); }
        Py_DECREF(entry);
      }
    }
    PyObject* count = PyLong_FromSsize_t(m);
    if (!count) return fail();
    PyList_SET_ITEM(counts, i, count);
  }
  return Py_BuildValue("(NNNN)", columns, counts, sorted, foreign);
}

PyObject* last_fast_slots(PyObject*, PyObject*) { return PyLong_FromSsize_t(g_last_fast_slots); }

// binding_samples(samples, lo, hi) -> [{"phase": "measure", "graphics_clock_mhz": s.get(...),
// "memory_clock_mhz": s.get(...)} for s in samples[lo:hi]]: the clock binding of a trial's
// selected measure samples (plain dicts read directly, anything else through its get()).
// Runs of samples with equal clocks (same type and value) share one entry object.
PyObject* binding_samples(PyObject*, PyObject* args) {
  PyObject* samples;
  Py_ssize_t lo, hi;
  Py_buffer repeat{};
  if (!PyArg_ParseTuple(args, "O!nn|y*", &PyList_Type, &samples, &lo, &hi, &repeat)) return nullptr;
  struct Release { Py_buffer* b; ~Release() { if (b->obj) PyBuffer_Release(b); } } release_repeat{&repeat};
  const Py_ssize_t n = PyList_GET_SIZE(samples);
  lo = lo < 0 ? 0 : lo > n ? n : lo;
  hi = hi < lo ? lo : hi > n ? n : hi;
  // repeat[i] = 1: sample i's clocks read back as sample i-1's (the packer's clock_repeat column)
  const uint8_t* rep = repeat.obj && repeat.len == n ? static_cast<const uint8_t*>(repeat.buf) : nullptr;
  static PyObject* k_phase = PyUnicode_InternFromString("phase");
  static PyObject* k_measure = PyUnicode_InternFromString("measure");
  static PyObject* k_gfx = PyUnicode_InternFromString("graphics_clock_mhz");
  static PyObject* k_mem = PyUnicode_InternFromString("memory_clock_mhz");
  if (!k_phase || !k_measure || !k_gfx || !k_mem) return nullptr;
  PyObject* out = PyList_New(hi - lo);
  if (!out) return nullptr;
  // Consecutive samples usually hold the same clocks: an entry whose two values read back as
  // the previous entry's (same_value) is that entry's dict object again.
  PyObject *last = nullptr, *last_gfx = nullptr, *last_mem = nullptr;
  for (Py_ssize_t i = lo; i < hi; ++i) {
    if (last && rep && rep[i]) {             // the previous entry's values, without reading the sample
      PyList_SET_ITEM(out, i - lo, Py_NewRef(last));
      continue;
    }
    PyObject* s = PyList_GET_ITEM(samples, i);
    PyObject *gfx = nullptr, *mem = nullptr;
    if (PyDict_CheckExact(s)) {              // borrowed values of a plain dict
      gfx = PyDict_GetItemWithError(s, k_gfx);
      if (gfx || !PyErr_Occurred()) mem = PyDict_GetItemWithError(s, k_mem);
      Py_XINCREF(gfx);
      Py_XINCREF(mem);
      if (!gfx && !PyErr_Occurred()) gfx = Py_NewRef(Py_None);
      if (!mem && !PyErr_Occurred()) mem = Py_NewRef(Py_None);
    } else {                                 // anything else answers its own get()
      gfx = PyObject_CallMethod(s, "get", "O", k_gfx);
      if (gfx) mem = PyObject_CallMethod(s, "get", "O", k_mem);
    }
    if (!gfx || !mem) {
      Py_XDECREF(gfx);
      Py_XDECREF(mem);
      Py_DECREF(out);
      return nullptr;
    }
    if (last) {
      if (same_value(gfx, last_gfx) && same_value(mem, last_mem)) {
        Py_DECREF(gfx);
        Py_DECREF(mem);
        PyList_SET_ITEM(out, i - lo, Py_NewRef(last));
        continue;
      }
    }
    PyObject* d = _PyDict_NewPresized(3);
    const bool ok = d && PyDict_SetItem(d, k_phase, k_measure) == 0 && PyDict_SetItem(d, k_gfx, gfx) == 0 &&
                    PyDict_SetItem(d, k_mem, mem) == 0;
    Py_DECREF(gfx);
    Py_DECREF(mem);
    if (!ok) {
      Py_XDECREF(d);
      Py_DECREF(out);
      return nullptr;
    }
    PyList_SET_ITEM(out, i - lo, d);
    last = d;                                // borrowed: the list holds it
    last_gfx = PyDict_GetItem(d, k_gfx);
    last_mem = PyDict_GetItem(d, k_mem);
  }
  return out;
}

// ---------------------------------------------------------------------------
// epochs(arms, fallback) -> (status, counts, columns): the completion-epoch
// lists of every (trial, arm) in one call, by the reference's parsing rules
// (powermodeling/analysis.py:228-276 as powermodeling_b200/pack.py states
// them in _epochs): the list under "measure_epochs" (else "work_epochs"),
// None -> PM_EP_NONE, not a non-empty list -> PM_EP_INVALID_LIST, parsing
// stops at the first item that is not a dict (PM_EP_NON_DICT_AFTER, the items
// before it kept); start_s / end_s through _finite, else the host monotonic
// (else plain) nanosecond stamps / 1e9; operations, logical_bytes and
// reference_loop_slots NaN when not finite; counts_exact only when True.
// An arm that is not an exact dict, or whose list or items are not exact
// lists and dicts, is parsed by `fallback` (the Python statement), which
// returns (status, [tuples]).
namespace {

PyObject* g_epoch_keys[11];
enum { E_MEASURE, E_WORK, E_START_S, E_END_S, E_HOST_START, E_START_NS, E_HOST_END, E_END_NS, E_OPS, E_BYTES, E_SLOTS };

// dict.get(key) of an exact dict, borrowed (NULL: absent); -1 on error.
int dget(PyObject* d, int key, PyObject** out) {
  *out = PyDict_GetItemWithError(d, g_epoch_keys[key]);
  return (!*out && PyErr_Occurred()) ? -1 : 0;
}

// d.get(a, d.get(b)) as the reference writes it: the value under `a` when the key is present.
int dget_or(PyObject* d, int a, int b, PyObject** out) {
  if (dget(d, a, out) < 0) return -1;
  if (*out) return 0;
  return dget(d, b, out);
}

// One epoch time: _finite(seconds), else _finite(stamp) / 1e9, else NaN.
int epoch_time(PyObject* epoch, int seconds, int host_ns, int plain_ns, double* out) {
  PyObject* v;
  double x;
  if (dget(epoch, seconds, &v) < 0) return -1;
  int r = finite(v, &x);
  if (r < 0) return -1;
  if (r) { *out = x; return 0; }
  if (dget_or(epoch, host_ns, plain_ns, &v) < 0) return -1;
  r = finite(v, &x);
  if (r < 0) return -1;
  *out = r ? x / 1e9 : kNaN;
  return 0;
}

int epoch_value(PyObject* epoch, int key, double* out) {
  PyObject* v;
  double x;
  if (dget(epoch, key, &v) < 0) return -1;
  const int r = finite(v, &x);
  if (r < 0) return -1;
  *out = r ? x : kNaN;
  return 0;
}

}  // namespace

PyObject* epochs(PyObject*, PyObject* args) {
  PyObject *arms, *fallback;
  if (!PyArg_ParseTuple(args, "O!O", &PyList_Type, &arms, &fallback)) return nullptr;
  static PyObject* k_exact = PyUnicode_InternFromString("counts_exact");
  if (!k_exact) return nullptr;
  if (!g_epoch_keys[0]) {
    const char* names[11] = {"measure_epochs", "work_epochs", "start_s", "end_s", "host_monotonic_start_ns", "start_ns",
                             "host_monotonic_end_ns", "end_ns", "operations", "logical_bytes", "reference_loop_slots"};
    for (int i = 0; i < 11; ++i)
      if (!(g_epoch_keys[i] = PyUnicode_InternFromString(names[i]))) return nullptr;
  }
  const Py_ssize_t n = PyList_GET_SIZE(arms);
  std::vector<int32_t> status((size_t)n), counts((size_t)n);
  std::vector<double> cols[5];
  std::vector<uint8_t> exact;
  auto push = [&](double a, double b, double ops, double bytes, double slots, bool ex) {
    cols[0].push_back(a); cols[1].push_back(b); cols[2].push_back(ops); cols[3].push_back(bytes); cols[4].push_back(slots);
    exact.push_back(ex ? 1 : 0);
  };
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* bench = PyList_GET_ITEM(arms, i);
    const size_t before = exact.size();
    bool plain = PyDict_CheckExact(bench);
    PyObject* source = nullptr;
    if (plain && dget_or(bench, E_MEASURE, E_WORK, &source) < 0) return nullptr;
    if (plain && source && source != Py_None && PyList_Check(source)) {
      if (!PyList_CheckExact(source)) plain = false;
      for (Py_ssize_t k = 0; plain && k < PyList_GET_SIZE(source); ++k) {
        PyObject* e = PyList_GET_ITEM(source, k);
        if (PyDict_Check(e) && !PyDict_CheckExact(e)) plain = false;
        if (!PyDict_Check(e)) break;              // parsing stops here either way
      }
    }
    if (!plain) {                                  // the Python statement for this arm
      PyObject* r = PyObject_CallOneArg(fallback, bench);
      if (!r) return nullptr;
      PyObject *st = nullptr, *items = nullptr;
      if (!PyArg_ParseTuple(r, "OO", &st, &items) || !PyList_Check(items)) {
        Py_DECREF(r);
        if (!PyErr_Occurred()) PyErr_SetString(PyExc_TypeError, "epoch fallback must return (status, list)");
        return nullptr;
      }
      status[(size_t)i] = (int32_t)PyLong_AsLong(st);
      for (Py_ssize_t k = 0; k < PyList_GET_SIZE(items); ++k) {
        double v[5];
        int ex = 0;
        PyObject* t = PyList_GET_ITEM(items, k);
        if (!PyArg_ParseTuple(t, "dddddp", &v[0], &v[1], &v[2], &v[3], &v[4], &ex)) { Py_DECREF(r); return nullptr; }
        push(v[0], v[1], v[2], v[3], v[4], ex != 0);
      }
      Py_DECREF(r);
      if (PyErr_Occurred()) return nullptr;
      counts[(size_t)i] = (int32_t)(exact.size() - before);
      continue;
    }
    if (!source || source == Py_None) { status[(size_t)i] = PM_EP_NONE; counts[(size_t)i] = 0; continue; }
    if (!PyList_Check(source) || PyList_GET_SIZE(source) == 0) {
      status[(size_t)i] = PM_EP_INVALID_LIST; counts[(size_t)i] = 0; continue;
    }
    int32_t st = PM_EP_OK;
    for (Py_ssize_t k = 0; k < PyList_GET_SIZE(source); ++k) {
      PyObject* e = PyList_GET_ITEM(source, k);
      if (!PyDict_Check(e)) { st = PM_EP_NON_DICT_AFTER; break; }
      double a, b, ops, bytes, slots;
      if (epoch_time(e, E_START_S, E_HOST_START, E_START_NS, &a) < 0 ||
          epoch_time(e, E_END_S, E_HOST_END, E_END_NS, &b) < 0 || epoch_value(e, E_OPS, &ops) < 0 ||
          epoch_value(e, E_BYTES, &bytes) < 0 || epoch_value(e, E_SLOTS, &slots) < 0)
        return nullptr;
      PyObject* ex = PyDict_GetItemWithError(e, k_exact);
      if (!ex && PyErr_Occurred()) return nullptr;
      push(a, b, ops, bytes, slots, ex == Py_True);
    }
    status[(size_t)i] = st;
    counts[(size_t)i] = (int32_t)(exact.size() - before);
  }
  auto bytes_of = [](const void* p, size_t nbytes) { return PyByteArray_FromStringAndSize(static_cast<const char*>(p), (Py_ssize_t)nbytes); };
  PyObject* columns = PyTuple_New(6);
  if (!columns) return nullptr;
  for (int c = 0; c < 5; ++c) {
    PyObject* b = bytes_of(cols[c].data(), cols[c].size() * sizeof(double));
    if (!b) { Py_DECREF(columns); return nullptr; }
    PyTuple_SET_ITEM(columns, c, b);
  }
  PyObject* b = bytes_of(exact.data(), exact.size());
  if (!b) { Py_DECREF(columns); return nullptr; }
  PyTuple_SET_ITEM(columns, 5, b);
  return Py_BuildValue("(NNN)", bytes_of(status.data(), status.size() * 4), bytes_of(counts.data(), counts.size() * 4),
                       columns);
}

PyMethodDef kMethods[] = {
    {"pack", pack, METH_VARARGS, "pack(slots, pids, source_ids) -> (columns, counts, sorted, foreign)"},
    {"last_fast_slots", last_fast_slots, METH_NOARGS, "slots the last pack() call packed on its parallel fast path"},
    {"binding_samples", binding_samples, METH_VARARGS, "binding_samples(samples, lo, hi) -> measure clock bindings"},
    {"epochs", epochs, METH_VARARGS, "epochs(arms, fallback) -> (status, counts, columns) of every arm's epoch list"},
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
