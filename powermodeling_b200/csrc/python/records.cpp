// _recordnative: host-side helpers that assemble the summary's records from
// plain Python data, in C++ over the CPython object API.
//
// fold(values, fallback) is the group diagnostics' fold of the repeats'
// measurement diagnostics (the rule of powermodeling/analysis.py:567-595 as
// powermodeling_b200/trial_report.py states it in _fold):
//  * the first value that is not None decides the kind;
//  * dicts fold key by key over the union of their keys in first-seen order,
//    a repeat without the key (or without a dict) contributing None;
//  * lists become their distinct items, ordered by first appearance (the
//    last equal item is kept);
//  * bools fold to "every value is True"; str (exact) and None stay the first;
//  * anything else: the median of the finite int and float values (a stable
//    sort, the middle value or the mean of the middle two), else the first.
// Exact dicts, exact lists of exact str, exact floats and ints, bools, None
// and exact str are folded here; any other node (subclasses, list items that
// are not strings, numbers of other types) is handed to `fallback`, the
// Python statement of the same rule, with the node's values as a list, so
// both paths return the same objects.
//
// phase_dicts and measurement_diagnostics (below) build the trial records'
// phase dicts and measurement diagnostics; their Python statements in
// powermodeling_b200/analysis.py and trial_report.py are the specification.
// sorted_json writes the group key's JSON text (json.dumps with sorted keys).
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

// One node of the fold: borrowed values (NULL counts as None).
PyObject* fold_node(const std::vector<PyObject*>& values, PyObject* fallback);

PyObject* call_fallback(const std::vector<PyObject*>& values, PyObject* fallback) {
  PyObject* list = PyList_New((Py_ssize_t)values.size());
  if (!list) return nullptr;
  for (size_t i = 0; i < values.size(); ++i) {
    PyObject* v = values[i] ? values[i] : Py_None;
    PyList_SET_ITEM(list, (Py_ssize_t)i, Py_NewRef(v));
  }
  PyObject* out = PyObject_CallOneArg(fallback, list);
  Py_DECREF(list);
  return out;
}

PyObject* fold_dicts(const std::vector<PyObject*>& values, PyObject* fallback) {
  // every dict value must be exact: a subclass may answer iteration or get() its own way
  for (PyObject* v : values)
    if (v && PyDict_Check(v) && !PyDict_CheckExact(v)) return call_fallback(values, fallback);
  PyObject* keys = PyDict_New();          // the union of keys, first-seen order
  if (!keys) return nullptr;
  for (PyObject* v : values) {
    if (!v || !PyDict_CheckExact(v)) continue;
    Py_ssize_t pos = 0;
    PyObject *k, *x;
    while (PyDict_Next(v, &pos, &k, &x)) {
      if (PyDict_SetDefault(keys, k, Py_None) == nullptr) { Py_DECREF(keys); return nullptr; }
    }
  }
  PyObject* out = _PyDict_NewPresized(PyDict_GET_SIZE(keys));
  if (!out) { Py_DECREF(keys); return nullptr; }
  std::vector<PyObject*> column(values.size());
  Py_ssize_t pos = 0;
  PyObject *k, *unused;
  while (PyDict_Next(keys, &pos, &k, &unused)) {
    for (size_t i = 0; i < values.size(); ++i) {
      PyObject* v = values[i];
      PyObject* x = nullptr;
      if (v && PyDict_CheckExact(v)) {
        x = PyDict_GetItemWithError(v, k);
        if (!x && PyErr_Occurred()) { Py_DECREF(out); Py_DECREF(keys); return nullptr; }
      }
      column[i] = x;
    }
    PyObject* folded = fold_node(column, fallback);
    if (!folded || PyDict_SetItem(out, k, folded) < 0) {
      Py_XDECREF(folded);
      Py_DECREF(out);
      Py_DECREF(keys);
      return nullptr;
    }
    Py_DECREF(folded);
  }
  Py_DECREF(keys);
  return out;
}

PyObject* fold_lists(const std::vector<PyObject*>& values, PyObject* fallback) {
  // Distinct items by their JSON text; for exact str items that is string equality.
  for (PyObject* v : values) {
    if (!v || !PyList_Check(v)) continue;
    if (!PyList_CheckExact(v)) return call_fallback(values, fallback);
    for (Py_ssize_t i = 0; i < PyList_GET_SIZE(v); ++i)
      if (!PyUnicode_CheckExact(PyList_GET_ITEM(v, i))) return call_fallback(values, fallback);
  }
  PyObject* seen = PyDict_New();          // item -> last equal item, first-seen order
  if (!seen) return nullptr;
  for (PyObject* v : values) {
    if (!v || !PyList_CheckExact(v)) continue;
    for (Py_ssize_t i = 0; i < PyList_GET_SIZE(v); ++i) {
      PyObject* item = PyList_GET_ITEM(v, i);
      if (PyDict_SetItem(seen, item, item) < 0) { Py_DECREF(seen); return nullptr; }
    }
  }
  PyObject* out = PyDict_Values(seen);
  Py_DECREF(seen);
  return out;
}

PyObject* fold_numbers(const std::vector<PyObject*>& values, PyObject* first, PyObject* fallback) {
  std::vector<double> numbers;
  numbers.reserve(values.size());
  for (PyObject* v : values) {
    if (!v) continue;
    if (PyFloat_CheckExact(v)) {
      const double d = PyFloat_AS_DOUBLE(v);
      if (std::isfinite(d)) numbers.push_back(d);
    } else if (PyLong_CheckExact(v)) {
      const double d = PyLong_AsDouble(v);  // OverflowError as math.isfinite raises it
      if (d == -1.0 && PyErr_Occurred()) return nullptr;
      numbers.push_back(d);
    } else if (PyBool_Check(v)) {
      continue;
    } else if (PyLong_Check(v) || PyFloat_Check(v)) {
      return call_fallback(values, fallback);   // numeric subclasses: their own float()
    }
  }
  if (numbers.empty()) return Py_NewRef(first ? first : Py_None);
  std::stable_sort(numbers.begin(), numbers.end());
  const size_t n = numbers.size(), mid = n / 2;
  return PyFloat_FromDouble(n % 2 ? numbers[mid] : (numbers[mid - 1] + numbers[mid]) / 2);
}

PyObject* fold_node(const std::vector<PyObject*>& values, PyObject* fallback) {
  PyObject* first = nullptr;
  for (PyObject* v : values)
    if (v && v != Py_None) { first = v; break; }
  if (!first) return Py_NewRef(Py_None);
  if (PyDict_Check(first)) return fold_dicts(values, fallback);
  if (PyList_Check(first)) return fold_lists(values, fallback);
  if (PyBool_Check(first)) {
    for (PyObject* v : values)
      if (v != Py_True) return Py_NewRef(Py_False);
    return Py_NewRef(Py_True);
  }
  if (PyUnicode_CheckExact(first)) return Py_NewRef(first);
  return fold_numbers(values, first, fallback);
}

PyObject* fold(PyObject*, PyObject* args) {
  PyObject *values, *fallback;
  if (!PyArg_ParseTuple(args, "O!O", &PyList_Type, &values, &fallback)) return nullptr;
  std::vector<PyObject*> v((size_t)PyList_GET_SIZE(values));
  for (Py_ssize_t i = 0; i < PyList_GET_SIZE(values); ++i) v[(size_t)i] = PyList_GET_ITEM(values, i);
  return fold_node(v, fallback);
}

// ---------------------------------------------------------------------------
// phase_dicts: the _phase_stats dict of every (trial, phase) slot from the
// analysis kernel's phase rows (powermodeling/analysis.py:255-423 as
// powermodeling_b200/analysis.py states it in _phase_dict): NaN is None,
// the issue and warning strings are "<issue>:<phase>", keys in the
// reference's insertion order.

// Phase-row positions, in the order the caller passes them.
enum PhaseIndex {
  P_START, P_END, P_DURATION, P_MIDPOINT, P_SAMPLES, P_GAP_MEDIAN, P_GAP_MAX, P_ENERGY, P_INTEGRATED_POWER, P_POWER,
  P_MEMORY_ENERGY, P_MEMORY_POWER, P_COUNTER, P_DISAGREEMENT, P_DISTINCT_POWER, P_CHANGE_MEDIAN,
  P_GFX_MED, P_GFX_MIN, P_GFX_MAX, P_SM_MED, P_SM_MIN, P_SM_MAX, P_MEM_MED, P_MEM_MIN, P_MEM_MAX,
  P_TEMP_MED, P_TEMP_MIN, P_TEMP_MAX, P_INDEX_COUNT
};

struct PhaseKeys {
  PyObject *name, *issues, *warnings, *start, *end, *duration, *midpoint, *samples, *gap_median, *gap_max, *energy,
      *integrated, *power, *memory_energy, *memory_power, *counter, *disagreement, *distinct, *change, *cadence;
  PyObject* clock[4][3];   // graphics, sm, memory clock and temperature: median, _min, _max
};

bool intern_all(PhaseKeys& k) {
  static bool done = false;
  if (done) return true;
  const char* clock_names[4] = {"graphics_clock_mhz", "sm_clock_mhz", "memory_clock_mhz", "temperature_c"};
  struct { PyObject** slot; const char* text; } names[] = {
      {&k.name, "name"}, {&k.issues, "issues"}, {&k.warnings, "warnings"}, {&k.start, "start_s"}, {&k.end, "end_s"},
      {&k.duration, "duration_s"}, {&k.midpoint, "midpoint_s"}, {&k.samples, "samples"},
      {&k.gap_median, "sample_interval_median_s"}, {&k.gap_max, "max_sample_gap_s"},
      {&k.energy, "integrated_power_energy_j"}, {&k.integrated, "integrated_power_w"}, {&k.power, "power_w"},
      {&k.memory_energy, "memory_rail_energy_j"}, {&k.memory_power, "memory_power_w"},
      {&k.counter, "energy_counter_j"}, {&k.disagreement, "counter_power_disagreement_fraction"},
      {&k.distinct, "distinct_power_values"}, {&k.change, "observed_power_change_interval_median_s"},
      {&k.cadence, "power_update_cadence_note"}};
  for (auto& n : names)
    if (!(*n.slot = PyUnicode_InternFromString(n.text))) return false;
  for (int f = 0; f < 4; ++f) {
    k.clock[f][0] = PyUnicode_InternFromString(clock_names[f]);
    k.clock[f][1] = PyUnicode_FromFormat("%s_min", clock_names[f]);
    k.clock[f][2] = PyUnicode_FromFormat("%s_max", clock_names[f]);
    if (!k.clock[f][0] || !k.clock[f][1] || !k.clock[f][2]) return false;
    PyUnicode_InternInPlace(&k.clock[f][1]);
    PyUnicode_InternInPlace(&k.clock[f][2]);
  }
  done = true;
  return true;
}

PhaseKeys g_phase_keys;

// A phase value as Python: None for NaN.
inline PyObject* value_or_none(double x) { return std::isnan(x) ? Py_NewRef(Py_None) : PyFloat_FromDouble(x); }

// Sets d[key] = value and releases value; false on error.
inline bool put(PyObject* d, PyObject* key, PyObject* value) {
  if (!value) return false;
  const int rc = PyDict_SetItem(d, key, value);
  Py_DECREF(value);
  return rc == 0;
}

// int(x) of a float64 as Python does it (truncation; ValueError for NaN, OverflowError for inf).
PyObject* int_of(double x) {
  PyObject* f = PyFloat_FromDouble(x);
  if (!f) return nullptr;
  PyObject* i = PyNumber_Long(f);
  Py_DECREF(f);
  return i;
}

// "<text>:<name>" appended to list.
inline bool append_issue(PyObject* list, PyObject* text, PyObject* name) {
  PyObject* s = PyUnicode_FromFormat("%U:%U", text, name);
  if (!s) return false;
  const int rc = PyList_Append(list, s);
  Py_DECREF(s);
  return rc == 0;
}

// phase_dicts(phase_out, phase_flags, width, names, index, bits, issue_bits, note) -> list of dicts
//   phase_out: float64 buffer, one row of `width` values per slot; phase_flags: uint32 per slot
//   names: the phase names, slot s is phase s % len(names)
//   index: the P_INDEX_COUNT row positions (PhaseIndex order)
//   bits: (missing, invalid window, counter reset) flag bits
//   issue_bits: ((bit, text), ...) in report order; note: the cadence note
PyObject* phase_dicts(PyObject*, PyObject* args) {
  Py_buffer po_buf, fl_buf;
  Py_ssize_t width;
  PyObject *names, *index, *bits, *issue_bits, *note;
  if (!PyArg_ParseTuple(args, "y*y*nO!O!O!O!U", &po_buf, &fl_buf, &width, &PyTuple_Type, &names, &PyTuple_Type, &index,
                        &PyTuple_Type, &bits, &PyTuple_Type, &issue_bits, &note))
    return nullptr;
  struct Release {
    Py_buffer *a, *b;
    ~Release() { PyBuffer_Release(a); PyBuffer_Release(b); }
  } release{&po_buf, &fl_buf};
  PhaseKeys& K = g_phase_keys;
  if (!intern_all(K)) return nullptr;
  const Py_ssize_t n_names = PyTuple_GET_SIZE(names);
  if (width <= 0 || n_names <= 0 || PyTuple_GET_SIZE(index) != P_INDEX_COUNT || PyTuple_GET_SIZE(bits) != 3) {
    PyErr_SetString(PyExc_ValueError, "phase_dicts: bad layout arguments");
    return nullptr;
  }
  const Py_ssize_t n_slots = fl_buf.len / (Py_ssize_t)sizeof(uint32_t);
  if (po_buf.len != n_slots * width * (Py_ssize_t)sizeof(double)) {
    PyErr_SetString(PyExc_ValueError, "phase_dicts: phase rows and flags differ in count");
    return nullptr;
  }
  int ix[P_INDEX_COUNT];
  for (int i = 0; i < P_INDEX_COUNT; ++i) {
    const long v = PyLong_AsLong(PyTuple_GET_ITEM(index, i));
    if (v == -1 && PyErr_Occurred()) return nullptr;
    if (v < 0 || v >= width) { PyErr_SetString(PyExc_ValueError, "phase_dicts: index outside the row"); return nullptr; }
    ix[i] = (int)v;
  }
  long fb[3];
  for (int i = 0; i < 3; ++i) {
    fb[i] = PyLong_AsLong(PyTuple_GET_ITEM(bits, i));
    if (fb[i] == -1 && PyErr_Occurred()) return nullptr;
  }
  const Py_ssize_t n_issues = PyTuple_GET_SIZE(issue_bits);
  std::vector<long> ibit((size_t)n_issues);
  std::vector<PyObject*> itext((size_t)n_issues);
  for (Py_ssize_t i = 0; i < n_issues; ++i) {
    PyObject* pair = PyTuple_GET_ITEM(issue_bits, i);
    if (!PyTuple_Check(pair) || PyTuple_GET_SIZE(pair) != 2) {
      PyErr_SetString(PyExc_ValueError, "phase_dicts: issue_bits holds (bit, text) pairs");
      return nullptr;
    }
    ibit[(size_t)i] = PyLong_AsLong(PyTuple_GET_ITEM(pair, 0));
    if (ibit[(size_t)i] == -1 && PyErr_Occurred()) return nullptr;
    itext[(size_t)i] = PyTuple_GET_ITEM(pair, 1);
  }
  static PyObject* s_missing = PyUnicode_InternFromString("missing_phase");
  static PyObject* s_invalid = PyUnicode_InternFromString("invalid_phase_window");
  static PyObject* s_reset = PyUnicode_InternFromString("energy_counter_reset");
  if (!s_missing || !s_invalid || !s_reset) return nullptr;
  const double* po_all = static_cast<const double*>(po_buf.buf);
  const uint32_t* flags_all = static_cast<const uint32_t*>(fl_buf.buf);
  PyObject* out = PyList_New(n_slots);
  if (!out) return nullptr;
  for (Py_ssize_t s = 0; s < n_slots; ++s) {
    const double* po = po_all + s * width;
    const uint32_t flags = flags_all[s];
    PyObject* name = PyTuple_GET_ITEM(names, s % n_names);
    PyObject* d = _PyDict_NewPresized(32);
    if (!d) { Py_DECREF(out); return nullptr; }
    PyList_SET_ITEM(out, s, d);
    PyObject* issues = PyList_New(0);
    PyObject* warnings = PyList_New(0);
    auto fail = [&]() -> PyObject* { Py_XDECREF(issues); Py_XDECREF(warnings); Py_DECREF(out); return nullptr; };
    if (!issues || !warnings || PyDict_SetItem(d, K.name, name) < 0 || PyDict_SetItem(d, K.issues, issues) < 0 ||
        PyDict_SetItem(d, K.warnings, warnings) < 0)
      return fail();
    Py_DECREF(issues);                 // borrowed from d from here on
    Py_DECREF(warnings);
    auto bad = [&]() -> PyObject* { Py_DECREF(out); return nullptr; };
    if (flags >> fb[0] & 1u) {
      if (!append_issue(issues, s_missing, name)) return bad();
      continue;
    }
    if (flags >> fb[1] & 1u) {
      if (!append_issue(issues, s_invalid, name)) return bad();
      continue;
    }
    if (!put(d, K.start, value_or_none(po[ix[P_START]])) || !put(d, K.end, value_or_none(po[ix[P_END]])) ||
        !put(d, K.duration, value_or_none(po[ix[P_DURATION]])) ||
        !put(d, K.midpoint, value_or_none(po[ix[P_MIDPOINT]])) || !put(d, K.samples, int_of(po[ix[P_SAMPLES]])) ||
        !put(d, K.gap_median, value_or_none(po[ix[P_GAP_MEDIAN]])) ||
        !put(d, K.gap_max, value_or_none(po[ix[P_GAP_MAX]])))
      return bad();
    for (Py_ssize_t i = 0; i < n_issues; ++i)
      if (flags >> ibit[(size_t)i] & 1u)
        if (!append_issue(issues, itext[(size_t)i], name)) return bad();
    if (!put(d, K.energy, value_or_none(po[ix[P_ENERGY]])) ||
        !put(d, K.integrated, value_or_none(po[ix[P_INTEGRATED_POWER]])) ||
        !put(d, K.power, value_or_none(po[ix[P_POWER]])) ||
        !put(d, K.memory_energy, value_or_none(po[ix[P_MEMORY_ENERGY]])) ||
        !put(d, K.memory_power, value_or_none(po[ix[P_MEMORY_POWER]])))
      return bad();
    if ((flags >> fb[2] & 1u) && !append_issue(warnings, s_reset, name)) return bad();
    if (!put(d, K.counter, value_or_none(po[ix[P_COUNTER]]))) return bad();
    if (!std::isnan(po[ix[P_DISAGREEMENT]]) && !put(d, K.disagreement, PyFloat_FromDouble(po[ix[P_DISAGREEMENT]])))
      return bad();
    if (!put(d, K.distinct, int_of(po[ix[P_DISTINCT_POWER]])) ||
        !put(d, K.change, value_or_none(po[ix[P_CHANGE_MEDIAN]])) || PyDict_SetItem(d, K.cadence, note) < 0)
      return bad();
    for (int f = 0; f < 4; ++f)
      for (int j = 0; j < 3; ++j)
        if (!put(d, K.clock[f][j], value_or_none(po[ix[P_GFX_MED + 3 * f + j]]))) return bad();
  }
  return out;
}

// ---------------------------------------------------------------------------
// measurement_diagnostics: a trial's measurement diagnostics (the rules of
// powermodeling/analysis.py:530-566 as powermodeling_b200/trial_report.py
// states them in measurement_diagnostics, which stays the specification):
// each objective's reported pJ beside its reconstruction from energy and
// count (or power and rate), scope factors, power shares, telemetry and
// throughput cross-checks, execution facts and timing, keys in that
// function's order.  Values read from the records are the records' own
// objects; sums of epoch durations go through Python's sum().

// _finite: 1 and *out when finite, 0 for None, a bool or a value float()
// rejects, -1 with an exception set (float()'s other errors).
int py_finite(PyObject* v, double* out) {
  if (!v || v == Py_None || PyBool_Check(v)) return 0;
  double d;
  if (PyFloat_CheckExact(v)) {
    d = PyFloat_AS_DOUBLE(v);
  } else if (PyLong_CheckExact(v)) {
    d = PyLong_AsDouble(v);
    if (d == -1.0 && PyErr_Occurred()) return -1;
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

// An optional float of the diagnostics.
struct Opt {
  bool has = false;
  double v = 0.0;
  PyObject* py() const { return has ? PyFloat_FromDouble(v) : Py_NewRef(Py_None); }
};
inline Opt some(double v) { return Opt{true, v}; }

// An interned key per string literal (cached by the literal's address).
PyObject* key_of(const char* text) {
  static std::unordered_map<const char*, PyObject*> cache;
  auto it = cache.find(text);
  if (it != cache.end()) return it->second;
  PyObject* k = PyUnicode_InternFromString(text);
  if (k) cache.emplace(text, k);
  return k;
}

// m.get(key[, default]) as a new reference: exact dicts directly, anything else through its get().
PyObject* get_new(PyObject* m, const char* key, PyObject* dflt = Py_None) {
  PyObject* k = key_of(key);
  if (!k) return nullptr;
  if (PyDict_CheckExact(m)) {
    PyObject* v = PyDict_GetItemWithError(m, k);
    if (!v) return PyErr_Occurred() ? nullptr : Py_NewRef(dflt);
    return Py_NewRef(v);
  }
  return PyObject_CallMethodObjArgs(m, key_of("get"), k, dflt, nullptr);
}

// m.get(key) for a key built at run time (not cached), as a new reference.
PyObject* get_dynamic(PyObject* m, const std::string& key) {
  PyObject* k = PyUnicode_FromStringAndSize(key.data(), (Py_ssize_t)key.size());
  if (!k) return nullptr;
  PyObject* v;
  if (PyDict_CheckExact(m)) {
    v = PyDict_GetItemWithError(m, k);
    v = v ? Py_NewRef(v) : (PyErr_Occurred() ? nullptr : Py_NewRef(Py_None));
  } else {
    v = PyObject_CallMethodObjArgs(m, key_of("get"), k, nullptr);
  }
  Py_DECREF(k);
  return v;
}

// _finite(m.get(key)) into *out; -1 with an exception set.
int finite_of(PyObject* m, const char* key, Opt* out) {
  PyObject* v = get_new(m, key);
  if (!v) return -1;
  double d;
  const int r = py_finite(v, &d);
  Py_DECREF(v);
  if (r < 0) return -1;
  *out = r ? some(d) : Opt{};
  return 0;
}

// m.get(key) is True
int is_true(PyObject* m, const char* key, bool* out) {
  PyObject* v = get_new(m, key);
  if (!v) return -1;
  *out = v == Py_True;
  Py_DECREF(v);
  return 0;
}

inline Opt ratio(Opt a, Opt b) { return a.has && b.has && b.v > 0 ? some(a.v / b.v) : Opt{}; }

// A dict built in key order; any failure leaves `ok` false and the exception set.
struct DictBuilder {
  PyObject* d;
  bool ok;
  DictBuilder() : d(PyDict_New()), ok(d != nullptr) {}
  ~DictBuilder() { Py_XDECREF(d); }
  DictBuilder& set(const char* key, PyObject* value) {          // steals `value`
    if (!ok || !value) { ok = false; Py_XDECREF(value); return *this; }
    PyObject* k = key_of(key);
    ok = k && PyDict_SetItem(d, k, value) == 0;
    Py_DECREF(value);
    return *this;
  }
  DictBuilder& ref(const char* key, PyObject* value) { return set(key, Py_NewRef(value ? value : Py_None)); }
  DictBuilder& from(const char* key, PyObject* m, const char* field) { return set(key, ok ? get_new(m, field) : nullptr); }
  DictBuilder& str(const char* key, const char* text) { return set(key, text ? PyUnicode_FromString(text) : Py_NewRef(Py_None)); }
  DictBuilder& num(const char* key, Opt v) { return set(key, v.py()); }
  DictBuilder& flag(const char* key, bool v) { return set(key, PyBool_FromLong(v)); }
  PyObject* take() { if (!ok) return nullptr; PyObject* r = d; d = nullptr; return r; }
};

// The workload classes the diagnostics distinguish (the caller's sets).
struct Classes {
  PyObject *memory, *tensor, *sfu, *nonlinear;
};

int member(PyObject* set, PyObject* workload, bool* out) {
  const int r = PySet_Contains(set, workload);
  if (r < 0) return -1;
  *out = r == 1;
  return 0;
}

// The work denominator: unit, energy-metric suffix, rate per second, selected count.
struct Denominator {
  const char *unit = nullptr, *suffix = nullptr;
  Opt rate, count;
};

int denominator(PyObject* result, PyObject* workload, const Classes& C, Denominator* d) {
  bool memory, sfu, tensor, nonlinear;
  if (member(C.memory, workload, &memory) < 0) return -1;
  if (memory) {
    Opt rate, count;
    if (finite_of(result, "throughput_bytes_s", &rate) < 0 || finite_of(result, "counted_measure_logical_bytes", &count) < 0)
      return -1;
    d->unit = "logical bit";
    d->suffix = "pj_per_logical_bit";
    d->rate = rate.has ? some(rate.v * 8) : Opt{};
    d->count = count.has ? some(count.v * 8) : Opt{};
    return 0;
  }
  if (member(C.sfu, workload, &sfu) < 0 || member(C.tensor, workload, &tensor) < 0 ||
      member(C.nonlinear, workload, &nonlinear) < 0)
    return -1;
  if (sfu || tensor || nonlinear) {
    d->unit = sfu ? "scalar SFU instruction" : tensor ? "FLOP" : "element";
    d->suffix = sfu ? "pj_per_instruction" : tensor ? "pj_per_flop" : "pj_per_element";
    if (finite_of(result, "throughput_ops_s", &d->rate) < 0 || finite_of(result, "counted_measure_operations", &d->count) < 0)
      return -1;
  }
  return 0;
}

PyObject* objective(PyObject* result, const char* name, const char* prefix, const char* power_field,
                    const char* energy_field, const Denominator& D, bool exact) {
  const bool total = strcmp(name, "total") == 0;
  bool eligible;
  if (total) {
    bool valid;
    if (is_true(result, "valid", &valid) < 0) return nullptr;
    eligible = valid && exact;
  } else {
    PyObject* v = get_dynamic(result, std::string(name) + "_eligible");
    if (!v) return nullptr;
    eligible = v == Py_True;
    Py_DECREF(v);
  }
  Opt power, energy, reported;
  if (finite_of(result, power_field, &power) < 0 || finite_of(result, energy_field, &energy) < 0) return nullptr;
  std::string metric = D.suffix ? std::string(prefix) + D.suffix : std::string();
  if (D.suffix) {
    PyObject* v = get_dynamic(result, metric);
    if (!v) return nullptr;
    double x;
    const int r = py_finite(v, &x);
    Py_DECREF(v);
    if (r < 0) return nullptr;
    reported = r ? some(x) : Opt{};
  }
  Opt rebuilt = exact ? ratio(energy, D.count) : ratio(power, D.rate);
  if (rebuilt.has) rebuilt.v = rebuilt.v * 1e12;
  DictBuilder b;
  b.set("metric", D.suffix ? PyUnicode_FromString(metric.c_str()) : Py_NewRef(Py_None));
  b.set("unit", D.unit ? PyUnicode_FromFormat("pJ/%s", D.unit) : Py_NewRef(Py_None));
  b.num("reported_value", reported).num("reconstructed_value", rebuilt);
  b.num("reconstruction_difference", reported.has && rebuilt.has ? some(reported.v - rebuilt.v) : Opt{});
  b.num("power_w", power).num("energy_j", energy).flag("eligible", eligible);
  b.str("scope", total ? "whole-device total"
                       : "whole-device operational contrast; physical component energy is not isolated");
  return b.take();
}

PyObject* alias_entry(const char* canonical, PyObject* multiplier, PyObject* unit) {   // steals both
  DictBuilder b;
  b.str("canonical_metric", canonical).set("value_multiplier", multiplier).set("unit", unit);
  return b.take();
}

PyObject* aliases(PyObject* result, PyObject* bench, PyObject* workload, const Classes& C, const Denominator& D) {
  bool memory, tensor, nonlinear;
  if (member(C.memory, workload, &memory) < 0) return nullptr;
  DictBuilder b;
  if (memory) {
    Opt ops, nbytes;
    if (finite_of(result, "counted_measure_operations", &ops) < 0 ||
        finite_of(result, "counted_measure_logical_bytes", &nbytes) < 0)
      return nullptr;
    const Opt per_op = ratio(nbytes.has ? some(nbytes.v * 8) : Opt{}, ops);
    PyObject* dflt = PyUnicode_FromString("pJ/reported memory operation");
    PyObject* unit = dflt ? get_new(bench, "operation_unit", dflt) : nullptr;
    Py_XDECREF(dflt);
    b.set("pj_per_logical_byte", alias_entry("operational_idle_increment_pj_per_logical_bit", PyLong_FromLong(8),
                                             PyUnicode_FromString("pJ/logical byte")));
    b.set("total_pj_per_logical_byte", alias_entry("total_pj_per_logical_bit", PyLong_FromLong(8),
                                                   PyUnicode_FromString("pJ/logical byte")));
    b.set("pj_per_op", unit ? alias_entry("operational_idle_increment_pj_per_logical_bit", per_op.py(), unit) : nullptr);
    return b.take();
  }
  if (member(C.tensor, workload, &tensor) < 0 || member(C.nonlinear, workload, &nonlinear) < 0) return nullptr;
  if (tensor || nonlinear) {
    b.set("pj_per_op", alias_entry(("operational_idle_increment_" + std::string(D.suffix)).c_str(), PyLong_FromLong(1),
                                   PyUnicode_FromFormat("pJ/%s", D.unit)));
    b.set("total_pj_per_op", alias_entry(("total_" + std::string(D.suffix)).c_str(), PyLong_FromLong(1),
                                         PyUnicode_FromFormat("pJ/%s", D.unit)));
  }
  return b.take();
}

// e[key] (any mapping), new reference.
PyObject* item(PyObject* e, const char* key) {
  PyObject* k = key_of(key);
  return k ? PyObject_GetItem(e, k) : nullptr;
}

// The epoch timing figures: durations' sum, span, summed readback seconds (None: absent).
struct EpochTiming {
  PyObject *span = nullptr, *summed = nullptr, *gap = nullptr;   // new references or NULL for None
  Opt readback_s;
  ~EpochTiming() { Py_XDECREF(span); Py_XDECREF(summed); Py_XDECREF(gap); }
};

int epoch_timing(PyObject* epochs, PyObject* sum_fn, EpochTiming* T) {
  const Py_ssize_t n = PyList_GET_SIZE(epochs);
  if (n == 0) return 0;
  PyObject* durations = PyList_New(n);
  PyObject* readbacks = PyList_New(n);
  if (!durations || !readbacks) { Py_XDECREF(durations); Py_XDECREF(readbacks); return -1; }
  bool all_ok = true;
  for (Py_ssize_t i = 0; i < n; ++i) {
    PyObject* e = PyList_GET_ITEM(epochs, i);
    PyObject* a = item(e, "start_s");
    PyObject* b = a ? item(e, "end_s") : nullptr;
    PyObject* d = b ? PyNumber_Subtract(b, a) : nullptr;
    Py_XDECREF(a);
    Py_XDECREF(b);
    if (!d) { Py_DECREF(durations); Py_DECREF(readbacks); return -1; }
    PyList_SET_ITEM(durations, i, d);
    Opt r;
    if (finite_of(e, "counter_readback_ns", &r) < 0) { Py_DECREF(durations); Py_DECREF(readbacks); return -1; }
    if (!r.has || !(r.v >= 0)) all_ok = false;
    PyList_SET_ITEM(readbacks, i, r.py());
  }
  PyObject* first = PyList_GET_ITEM(epochs, 0);
  PyObject* last = PyList_GET_ITEM(epochs, n - 1);
  PyObject* end = item(last, "end_s");
  PyObject* start = end ? item(first, "start_s") : nullptr;
  T->span = start ? PyNumber_Subtract(end, start) : nullptr;
  Py_XDECREF(end);
  Py_XDECREF(start);
  T->summed = T->span ? PyObject_CallOneArg(sum_fn, durations) : nullptr;
  PyObject* rs = nullptr;
  if (T->summed && all_ok) {
    rs = PyObject_CallOneArg(sum_fn, readbacks);
    if (rs) {
      const double x = PyFloat_AsDouble(rs);
      if (!(x == -1.0 && PyErr_Occurred())) T->readback_s = some(x / 1e9);
    }
  }
  Py_DECREF(durations);
  Py_DECREF(readbacks);
  if (!T->summed || (all_ok && !rs) || PyErr_Occurred()) { Py_XDECREF(rs); return -1; }
  Py_XDECREF(rs);
  // max(0.0, span - summed)
  PyObject* diff = PyNumber_Subtract(T->span, T->summed);
  if (!diff) return -1;
  PyObject* zero = PyFloat_FromDouble(0.0);
  const int greater = zero ? PyObject_RichCompareBool(diff, zero, Py_GT) : -1;
  if (greater < 0) { Py_DECREF(diff); Py_XDECREF(zero); return -1; }
  T->gap = greater ? diff : zero;
  Py_DECREF(greater ? zero : diff);
  return 0;
}

PyObject* measurement_diagnostics(PyObject*, PyObject* args) {
  PyObject *result, *bench, *epochs, *sum_fn;
  Classes C;
  if (!PyArg_ParseTuple(args, "OOO!OOOOO", &result, &bench, &PyList_Type, &epochs, &C.memory, &C.tensor, &C.sfu,
                        &C.nonlinear, &sum_fn))
    return nullptr;
  PyObject* workload = get_new(result, "workload");
  if (!workload) return nullptr;
  bool memory = false, tensor = false;
  Denominator D;
  if (member(C.memory, workload, &memory) < 0 || member(C.tensor, workload, &tensor) < 0 ||
      denominator(result, workload, C, &D) < 0) {
    Py_DECREF(workload);
    return nullptr;
  }
  Opt duration, board, idle, reference, paired, incremental, integral, counter, ops, nbytes;
  bool exact = false;
  if (finite_of(result, "duration_s", &duration) < 0 || is_true(result, "count_energy_time_alignment_exact", &exact) < 0 ||
      finite_of(result, "board_power_w", &board) < 0 || finite_of(result, "idle_power_w", &idle) < 0 ||
      finite_of(result, "active_reference_power_w", &reference) < 0 ||
      finite_of(result, "paired_active_reference_power_w", &paired) < 0 ||
      finite_of(result, "operational_idle_increment_power_w", &incremental) < 0 ||
      finite_of(result, "integrated_power_energy_j", &integral) < 0 || finite_of(result, "energy_counter_j", &counter) < 0 ||
      finite_of(result, "counted_measure_operations", &ops) < 0 ||
      finite_of(result, "counted_measure_logical_bytes", &nbytes) < 0) {
    Py_DECREF(workload);
    return nullptr;
  }
  EpochTiming T;
  if (epoch_timing(epochs, sum_fn, &T) < 0) { Py_DECREF(workload); return nullptr; }
  bool idle_eligible, paired_eligible, target_verified, valid, baseline_valid;
  if (is_true(result, "operational_idle_increment_eligible", &idle_eligible) < 0 ||
      is_true(result, "paired_active_reference_eligible", &paired_eligible) < 0 ||
      is_true(result, "target_verified", &target_verified) < 0 || is_true(result, "valid", &valid) < 0 ||
      is_true(result, "baseline_valid", &baseline_valid) < 0) {
    Py_DECREF(workload);
    return nullptr;
  }

  DictBuilder den;
  den.str("unit", D.unit).num("measured_count", exact ? D.count : Opt{}).num("selected_epoch_count", D.count)
      .num("rate_per_s", D.rate).num("aligned_window_s", duration).flag("exact_matching_window", exact)
      .str("kind", exact ? "same-window counted work"
                         : "stationary whole-run throughput estimate; no exact energy-window work count");
  static const char* kObjectives[3][4] = {
      {"total", "total_", "board_power_w", "total_energy_j"},
      {"operational_idle_increment", "operational_idle_increment_", "operational_idle_increment_power_w",
       "operational_idle_increment_energy_j"},
      {"paired_active_reference", "paired_active_reference_", "paired_active_reference_power_w",
       "paired_active_reference_energy_j"}};
  DictBuilder obj;
  for (auto& o : kObjectives) obj.set(o[0], obj.ok ? objective(result, o[0], o[1], o[2], o[3], D, exact) : nullptr);
  DictBuilder units;
  units.set("bits_per_byte", memory ? PyLong_FromLong(8) : Py_NewRef(Py_None))
      .set("flops_per_fma", tensor ? PyLong_FromLong(2) : Py_NewRef(Py_None))
      .from("flop_convention", result, "flop_count_convention").from("reported_operation_unit", bench, "operation_unit")
      .num("logical_bits_per_reported_memory_operation", memory ? ratio(nbytes.has ? some(nbytes.v * 8) : Opt{}, ops) : Opt{})
      .str("logical_byte_scope", memory ? "requested read payload plus requested write payload for copy; not physical "
                                          "cache-sector or DRAM traffic" : nullptr)
      .set("aliases", units.ok ? aliases(result, bench, workload, C, D) : nullptr);
  DictBuilder scope;
  scope.num("total_over_idle_increment", ratio(board, incremental)).num("total_over_paired_reference", ratio(board, paired))
      .flag("idle_increment_eligible", idle_eligible).flag("paired_reference_eligible", paired_eligible)
      .str("interpretation", "Numerical operational scope ratios only; ineligible contrasts and component literature "
                             "must not be silently substituted.");
  DictBuilder power;
  power.num("total_w", board).num("idle_w", idle).num("idle_fraction", ratio(idle, board)).num("paired_reference_w", reference)
      .num("paired_reference_fraction", ratio(reference, board)).num("idle_increment_w", incremental)
      .num("paired_contrast_w", paired);
  DictBuilder tele;
  tele.from("energy_source", result, "energy_source").num("counter_energy_j", counter).num("integrated_power_energy_j", integral)
      .num("counter_over_integrated", ratio(counter, integral))
      .num("disagreement_fraction", counter.has && integral.has && integral.v > 0
                                        ? some(std::fabs(counter.v - integral.v) / integral.v) : Opt{});
  DictBuilder thr;
  thr.set("unit", D.unit ? PyUnicode_FromFormat("%s/s", D.unit) : Py_NewRef(Py_None)).num("sustained_rate_per_s", D.rate)
      .ref("profiler_replay_rate_per_s", nullptr).ref("profiler_replay_count", nullptr)
      .ref("profiler_replay_summed_kernel_duration_s", nullptr).ref("profiler_over_sustained_rate", nullptr)
      .flag("profiler_target_verified", target_verified).flag("same_energy_run", false)
      .str("note", "Profiler replay uses a different run and summed kernel duration. Rate disagreement can motivate "
                   "timing/traffic review but does not prove host overhead, permit energy rescaling or supply "
                   "same-window physical traffic.");
  DictBuilder exe;
  exe.from("kernel_resources", bench, "kernel_resources").from("sfu_contract", result, "sfu_contract")
      .from("sfu_reference_delta", result, "sfu_reference_delta_diagnostics")
      .from("auxiliary_work", bench, "auxiliary_work").from("execution_diagnostics", bench, "execution_diagnostics")
      .from("implementation_version", bench, "kernel_implementation_version");
  for (const char* k : {"memory_accesses_per_thread_iteration", "memory_read_checksum_scope", "memory_read_validation",
                        "grid_mode", "input_elements", "block_completion_count_source", "active_sm_ids",
                        "active_sm_distribution_status", "sm_distribution_scope"})
    exe.from(k, bench, k);
  exe.str("saturation_status", "CUDA occupancy bounds and grid size do not establish achieved utilization or hardware "
                               "saturation");
  Opt host_duration, event_duration, mean_batch;
  if (finite_of(bench, "host_duration_s", &host_duration) < 0 || finite_of(bench, "duration_s", &event_duration) < 0 ||
      finite_of(bench, "mean_batch_duration_s", &mean_batch) < 0) {
    Py_DECREF(workload);
    return nullptr;
  }
  PyObject* scope_default = PyUnicode_FromString("CUDA experiment window; summed kernel busy time is not established");
  DictBuilder tim;
  tim.num("host_duration_s", host_duration).num("event_duration_s", event_duration)
      .set("event_duration_scope", scope_default ? get_new(bench, "duration_scope", scope_default) : nullptr)
      .num("mean_batch_experiment_duration_s", mean_batch)
      .set("complete_epochs", PyLong_FromSsize_t(PyList_GET_SIZE(epochs))).ref("complete_epoch_span_s", T.span)
      .ref("summed_epoch_duration_s", T.summed).ref("inter_epoch_gap_s", T.gap).num("counter_readback_s", T.readback_s)
      .num("counter_readback_fraction", ratio(T.readback_s, duration)).ref("kernel_busy_time_s", nullptr)
      .str("note", "Host synchronization, launch and readback gaps remain in sustained experiment energy and "
                   "throughput. CUDA event-window rate is not a kernel-busy rate; NCU replay is a separate run.");
  Py_XDECREF(scope_default);
  PyObject* empty_issues = PyList_New(0);
  PyObject* empty_baseline = PyList_New(0);
  DictBuilder qual;
  qual.flag("valid", valid).set("issues", empty_issues ? get_new(result, "issues", empty_issues) : nullptr)
      .flag("baseline_valid", baseline_valid)
      .set("baseline_issues", empty_baseline ? get_new(result, "baseline_issues", empty_baseline) : nullptr)
      .flag("target_verified", target_verified);
  Py_XDECREF(empty_issues);
  Py_XDECREF(empty_baseline);
  Py_DECREF(workload);

  DictBuilder out;
  out.set("schema_version", PyLong_FromLong(1)).set("denominator", den.take()).set("objectives", obj.take())
      .set("unit_conventions", units.take()).set("scope_factors", scope.take()).set("power_contributions", power.take())
      .set("telemetry_crosscheck", tele.take()).set("throughput_crosscheck", thr.take()).set("execution", exe.take())
      .set("timing", tim.take()).set("quality", qual.take());
  return out.take();
}

// ---------------------------------------------------------------------------
// sorted_json(obj): json.dumps(obj, sort_keys=True, separators=(",", ":"))
// (the group key's text, whose sha256 seeds the group's resampling): None,
// true/false, ints and floats by their reprs (NaN, Infinity, -Infinity),
// strings with every character outside printable ASCII escaped (\uXXXX,
// surrogate pairs above U+FFFF), lists and tuples, dicts with their items
// sorted and non-string keys written as their JSON text after sorting.
// Anything else raises TypeError, as json does without a default.

void json_string(std::string& out, PyObject* s) {
  const Py_ssize_t n = PyUnicode_GET_LENGTH(s);
  const int kind = PyUnicode_KIND(s);
  const void* data = PyUnicode_DATA(s);
  static const char hex[] = "0123456789abcdef";
  out.push_back('"');
  auto unit = [&](unsigned u) {
    out += "\\u";
    out.push_back(hex[(u >> 12) & 15]); out.push_back(hex[(u >> 8) & 15]);
    out.push_back(hex[(u >> 4) & 15]); out.push_back(hex[u & 15]);
  };
  for (Py_ssize_t i = 0; i < n; ++i) {
    const Py_UCS4 c = PyUnicode_READ(kind, data, i);
    if (c >= ' ' && c <= '~' && c != '\\' && c != '"') { out.push_back((char)c); continue; }
    switch (c) {
      case '\\': out += "\\\\"; break;
      case '"': out += "\\\""; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c >= 0x10000) {
          const Py_UCS4 v = c - 0x10000;
          unit(0xd800 | ((v >> 10) & 0x3ff));
          unit(0xdc00 | (v & 0x3ff));
        } else {
          unit(c);
        }
    }
  }
  out.push_back('"');
}

// The repr of an int or float as json writes it (NaN and infinities by name).
int json_number(std::string& out, PyObject* v) {
  PyObject* r;
  if (PyFloat_Check(v)) {
    const double d = PyFloat_AS_DOUBLE(v);
    if (std::isnan(d)) { out += "NaN"; return 0; }
    if (std::isinf(d)) { out += d > 0 ? "Infinity" : "-Infinity"; return 0; }
    r = PyFloat_Type.tp_repr(v);
  } else {
    r = PyLong_Type.tp_repr(v);
  }
  if (!r) return -1;
  Py_ssize_t len;
  const char* text = PyUnicode_AsUTF8AndSize(r, &len);
  if (!text) { Py_DECREF(r); return -1; }
  out.append(text, (size_t)len);
  Py_DECREF(r);
  return 0;
}

int json_value(std::string& out, PyObject* v, int depth) {
  if (depth > 1000) { PyErr_SetString(PyExc_RecursionError, "maximum recursion depth exceeded in sorted_json"); return -1; }
  if (v == Py_None) { out += "null"; return 0; }
  if (v == Py_True) { out += "true"; return 0; }
  if (v == Py_False) { out += "false"; return 0; }
  if (PyUnicode_Check(v)) { json_string(out, v); return 0; }
  if (PyLong_Check(v) || PyFloat_Check(v)) return json_number(out, v);
  if (PyList_Check(v) || PyTuple_Check(v)) {
    PyObject* seq = PySequence_Fast(v, "sequence");
    if (!seq) return -1;
    out.push_back('[');
    for (Py_ssize_t i = 0; i < PySequence_Fast_GET_SIZE(seq); ++i) {
      if (i) out.push_back(',');
      if (json_value(out, PySequence_Fast_GET_ITEM(seq, i), depth + 1) < 0) { Py_DECREF(seq); return -1; }
    }
    out.push_back(']');
    Py_DECREF(seq);
    return 0;
  }
  if (PyDict_Check(v)) {
    PyObject* items = PyMapping_Items(v);
    if (!items || PyList_Sort(items) < 0) { Py_XDECREF(items); return -1; }
    out.push_back('{');
    for (Py_ssize_t i = 0; i < PyList_GET_SIZE(items); ++i) {
      PyObject* kv = PyList_GET_ITEM(items, i);
      PyObject* k = PyTuple_GET_ITEM(kv, 0);
      if (i) out.push_back(',');
      if (PyUnicode_Check(k)) {
        json_string(out, k);
      } else if (PyFloat_Check(k) || (PyLong_Check(k) && !PyBool_Check(k))) {
        std::string text;
        if (json_number(text, k) < 0) { Py_DECREF(items); return -1; }
        out.push_back('"'); out += text; out.push_back('"');
      } else if (k == Py_True || k == Py_False || k == Py_None) {
        out += k == Py_True ? "\"true\"" : k == Py_False ? "\"false\"" : "\"null\"";
      } else {
        PyErr_Format(PyExc_TypeError, "keys must be str, int, float, bool or None, not %.100s", Py_TYPE(k)->tp_name);
        Py_DECREF(items);
        return -1;
      }
      out.push_back(':');
      if (json_value(out, PyTuple_GET_ITEM(kv, 1), depth + 1) < 0) { Py_DECREF(items); return -1; }
    }
    out.push_back('}');
    Py_DECREF(items);
    return 0;
  }
  PyErr_Format(PyExc_TypeError, "Object of type %.100s is not JSON serializable", Py_TYPE(v)->tp_name);
  return -1;
}

PyObject* sorted_json(PyObject*, PyObject* obj) {
  std::string out;
  out.reserve(1024);
  if (json_value(out, obj, 0) < 0) return nullptr;
  return PyUnicode_FromStringAndSize(out.data(), (Py_ssize_t)out.size());
}

PyMethodDef kMethods[] = {
    {"sorted_json", sorted_json, METH_O, "sorted_json(obj) -> json.dumps(obj, sort_keys=True, separators=(',', ':'))"},
    {"fold", fold, METH_VARARGS, "fold(values, fallback) -> the repeats' diagnostics folded into one"},
    {"measurement_diagnostics", measurement_diagnostics, METH_VARARGS,
     "measurement_diagnostics(result, bench, epochs, memory, tensor, sfu, nonlinear, sum) -> a trial's diagnostics"},
    {"phase_dicts", phase_dicts, METH_VARARGS,
     "phase_dicts(phase_out, phase_flags, width, names, index, bits, issue_bits, note) -> a phase dict per slot"},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_recordnative",
                       "Assembly of the summary's trial and group records from plain Python data.", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__recordnative(void) { return PyModule_Create(&kModule); }
