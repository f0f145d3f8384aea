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
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <algorithm>
#include <cmath>
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

PyMethodDef kMethods[] = {
    {"fold", fold, METH_VARARGS, "fold(values, fallback) -> the repeats' diagnostics folded into one"},
    {"phase_dicts", phase_dicts, METH_VARARGS,
     "phase_dicts(phase_out, phase_flags, width, names, index, bits, issue_bits, note) -> a phase dict per slot"},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_recordnative",
                       "Assembly of the summary's trial and group records from plain Python data.", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__recordnative(void) { return PyModule_Create(&kModule); }
