// Output slot and issue-bit layout of the analysis kernels.
//
// Each list is an X-macro so the kernel, pm_layout() (name -> index lookup
// for bindings) and the tests see one definition.  Slot names follow the
// keys the reference's analysis.py writes for a phase (_phase_stats,
// analysis.py:127-207) and for a trial (analyze_trial, 597-1056).
#pragma once

// ---- per-phase double slots -------------------------------------------------
#define PM_PHASE_FIELDS(X) \
  X(START_S) X(END_S) X(DURATION_S) X(MIDPOINT_S) X(SAMPLES) \
  X(GAP_MEDIAN_S) X(GAP_MAX_S) \
  X(ENERGY_J) X(INTEGRATED_POWER_W) X(POWER_W) X(MEMORY_ENERGY_J) X(MEMORY_POWER_W) \
  X(COUNTER_J) X(DISAGREEMENT) X(DISTINCT_POWER) X(CHANGE_MEDIAN_S) \
  X(GFX_MED) X(GFX_MIN) X(GFX_MAX) X(SM_MED) X(SM_MIN) X(SM_MAX) \
  X(MEM_MED) X(MEM_MIN) X(MEM_MAX) X(TEMP_MED) X(TEMP_MIN) X(TEMP_MAX) \
  X(PLIMIT_MED) X(PLIMIT_MIN) X(PLIMIT_MAX) X(PLIMIT_NONE) X(PLIMIT_FIN) \
  X(ENF_MED) X(ENF_MIN) X(ENF_MAX) X(ENF_NONE) X(ENF_FIN) \
  X(PSTATE_MED) X(PSTATE_MIN) X(PSTATE_MAX) X(PSTATE_NONE) X(PSTATE_FIN) \
  X(SEL_LO) X(SEL_HI) X(COV_LO) X(COV_HI) X(THROTTLE_OR) X(MEM_SOURCES)

// ---- per-phase flag bits ------------------------------------------------------
#define PM_PHASE_FLAGS(X) \
  X(MISSING) X(INVALID_WINDOW) X(SHORT_PLATEAU) X(TOO_FEW_SAMPLES) X(TELEMETRY_GAP) \
  X(NEGATIVE_POWER) X(MISSING_POWER_COVERAGE) X(COUNTER_DISAGREEMENT) X(COUNTER_RESET) \
  X(ANY_SM_FINITE) X(TEMP_MISSING) X(GFX_NONPOS) X(MEM_NONPOS) X(SM_NONPOS) \
  X(THROTTLE_MISSING) X(THROTTLE_ACTIVE) X(FOREIGN_PID) X(NO_COMPUTE_INV) X(NO_GRAPHICS_INV) \
  X(MPS) X(PID_UNKNOWN) X(REF_FOREIGN) X(COMPUTED) X(ALIGNED) X(LARGE)

// ---- per-trial double slots ---------------------------------------------------
#define PM_TRIAL_FIELDS(X) \
  X(DURATION_S) X(BENCH_MEASURED_DURATION_S) X(BENCH_DEVICE_DURATION_S) \
  X(IDLE_POWER_W) X(IDLE_MEMORY_POWER_W) X(TOTAL_ENERGY_J) X(ENERGY_SOURCE_TRAPEZOID) \
  X(BOARD_POWER_W) X(IDLE_ENERGY_J) X(INCREMENTAL_ENERGY_J) X(INCREMENTAL_POWER_W) \
  X(OPS_RATE) X(BYTE_RATE) X(DEVICE_OPS_RATE) X(DEVICE_BYTE_RATE) \
  X(COUNTED_OPS) X(COUNTED_BYTES) X(EPOCHS) X(EXACT) \
  X(RAIL_ENERGY_J) X(RAIL_INCREMENTAL_J) X(RAIL_INCREMENTAL_W) \
  X(POWER_LIMIT_W) X(TENSOR_PEAK_TFLOPS) X(PEAK_CLOCK_IS_SM) X(TENSOR_UTILIZATION) \
  X(IDLE_FRAC_MEASURED) X(IDLE_FRAC_LIMIT) X(LIMIT_UTILIZATION) \
  X(PJ_PER_OP) X(PJ_PER_LOGICAL_BYTE) X(TOTAL_PJ_PER_OP) X(TOTAL_PJ_PER_LOGICAL_BYTE) \
  X(TOTAL_PJ_PER_FLOP) X(TOTAL_PJ_PER_BIT) X(INC_PJ_PER_FLOP) X(INC_PJ_PER_BIT) \
  X(BASE_CLOCK_MATCHED) X(BASE_TEMP_MATCHED) X(BASE_CAP_MATCHED) X(BASE_STATE_MATCHED) \
  X(BASE_SM_COMPARED) X(BASE_ENF_COMPARED) X(BASE_PSTATE_COMPARED) \
  X(DPRE_GFX) X(DPRE_MEM) X(DPRE_SM) X(DPRE_TEMP) X(DPRE_ENF) X(DPRE_PSTATE) \
  X(DPOST_GFX) X(DPOST_MEM) X(DPOST_SM) X(DPOST_TEMP) X(DPOST_ENF) X(DPOST_PSTATE) \
  X(PAIRED_POWER_W) X(PAIRED_ENERGY_J) X(PAIRED_ELIGIBLE) \
  X(REF_POWER_W) X(REF_DURATION_S) X(REF_TOTAL_ENERGY_J) \
  X(PAIRED_PJ_PER_FLOP) X(PAIRED_PJ_PER_BIT) X(PAIRED_DRIFT_ADJUSTED_W) \
  X(PAIRED_D_GFX) X(PAIRED_D_MEM) X(PAIRED_D_SM) X(PAIRED_D_TEMP) X(PAIRED_SM_COMPARED) \
  X(REF_EPOCHS) X(REF_EXACT) X(REF_SLOTS) X(REF_SLOTS_RATE) \
  X(SFU_RATE) X(SFU_COUNTED) X(SFU_TOTAL_PJ) X(SFU_INC_PJ) X(SFU_PAIRED_PJ) \
  X(ELEMENT_RATE) X(ROW_RATE) X(COUNTED_ELEMENTS) \
  X(PJ_ELEMENT_TOTAL) X(PJ_ELEMENT_INC) X(PJ_ELEMENT_PAIRED) \
  X(PJ_ROW_TOTAL) X(PJ_ROW_INC) X(PJ_ROW_PAIRED) \
  X(CONTROL_INC_POWER_W) \
  X(VALID) X(BASELINE_VALID) X(IDLE_INC_ELIGIBLE) X(THROTTLE_MASK)

// ---- issue bits: word 0 treatment issues ------------------------------------
#define PM_ISSUES_TREATMENT(X) \
  X(M_MISSING_PHASE) X(M_INVALID_WINDOW) X(M_SHORT_PLATEAU) X(M_TOO_FEW_SAMPLES) X(M_TELEMETRY_GAP) \
  X(M_NEGATIVE_POWER) X(M_MISSING_POWER_COVERAGE) X(M_COUNTER_DISAGREEMENT) \
  X(EP_PHASE_WINDOW) X(EP_BOUNDARIES) X(EP_COUNT_OPERATIONS) X(EP_COUNT_LOGICAL_BYTES) \
  X(EP_OVERLAPPING) X(EP_INSUFFICIENT) X(EP_TOTAL_OPERATIONS) X(EP_TOTAL_LOGICAL_BYTES) X(EP_NON_DICT) \
  X(MISSING_CLOCK_GFX) X(MISSING_CLOCK_MEM) X(MISSING_CLOCK_SM) \
  X(CLOCK_MISMATCH_GFX) X(CLOCK_MISMATCH_MEM) X(CLOCK_MISMATCH_SM) \
  X(CLOCK_DRIFT_GFX) X(CLOCK_DRIFT_MEM) X(CLOCK_DRIFT_SM) \
  X(TEMPERATURE_DRIFT) X(MISSING_TEMPERATURE) X(MISSING_THROTTLING) X(ACTIVE_THROTTLING) \
  X(MISSING_INV_COMPUTE) X(MISSING_INV_GRAPHICS) X(MISSING_MEASUREMENT_PID) X(OTHER_GPU_PROCESSES) X(MPS_ACTIVE) \
  X(DURATION_DISAGREEMENT) X(MISSING_BENCH_DURATION) X(MISSING_OPERATION_COUNT) X(MISSING_LOGICAL_BYTE_COUNT) \
  X(NONLINEAR_EPOCHS) X(SFU_EPOCHS)

// ---- word 1 baseline issues -----------------------------------------------------
#define PM_ISSUES_BASELINE(X) \
  X(PRE_MISSING_PHASE) X(PRE_INVALID_WINDOW) X(PRE_SHORT_PLATEAU) X(PRE_TOO_FEW_SAMPLES) X(PRE_TELEMETRY_GAP) \
  X(PRE_NEGATIVE_POWER) X(PRE_MISSING_POWER_COVERAGE) X(PRE_COUNTER_DISAGREEMENT) \
  X(POST_MISSING_PHASE) X(POST_INVALID_WINDOW) X(POST_SHORT_PLATEAU) X(POST_TOO_FEW_SAMPLES) X(POST_TELEMETRY_GAP) \
  X(POST_NEGATIVE_POWER) X(POST_MISSING_POWER_COVERAGE) X(POST_COUNTER_DISAGREEMENT) \
  X(IDLE_DRIFT) X(MISSING_IDLE) X(NEGATIVE_INCREMENTAL) \
  X(B_MISSING_INV_COMPUTE) X(B_MISSING_INV_GRAPHICS) X(B_MISSING_MEASUREMENT_PID) X(B_OTHER_GPU_PROCESSES) X(B_MPS_ACTIVE) \
  X(STATE_PRE_ENF) X(STATE_PRE_PSTATE) X(STATE_POST_ENF) X(STATE_POST_PSTATE)

// ---- word 2 paired-reference issues -----------------------------------------------
#define PM_ISSUES_PAIRED(X) \
  X(R_MISSING_PHASE) X(R_INVALID_WINDOW) X(R_SHORT_PLATEAU) X(R_TOO_FEW_SAMPLES) X(R_TELEMETRY_GAP) \
  X(R_NEGATIVE_POWER) X(R_MISSING_POWER_COVERAGE) X(R_COUNTER_DISAGREEMENT) \
  X(REP_PHASE_WINDOW) X(REP_BOUNDARIES) X(REP_COUNT_OPERATIONS) X(REP_COUNT_LOGICAL_BYTES) \
  X(REP_OVERLAPPING) X(REP_INSUFFICIENT) X(REP_TOTAL_OPERATIONS) X(REP_TOTAL_LOGICAL_BYTES) X(REP_NON_DICT) \
  X(REF_WINDOW_UNVERIFIED) \
  X(STATE_GFX) X(STATE_MEM) X(STATE_SM) X(STATE_TEMP) \
  X(REF_THROTTLE) X(REF_INV_COMPUTE) X(REF_INV_GRAPHICS) X(REF_FOREIGN) \
  X(CAP_UNVERIFIED) X(CAP_CHANGED) X(STATE_ENF) X(STATE_PSTATE) \
  X(POWER_UNAVAILABLE) X(NONPOSITIVE_CONTRAST) X(MISSING_REFERENCE_PHASE)

// ---- word 3 warnings --------------------------------------------------------
#define PM_WARNINGS(X) \
  X(COUNTER_RESET_PRE) X(COUNTER_RESET_MEASURE) X(COUNTER_RESET_POST) X(COUNTER_RESET_CONTROL) \
  X(UNCONTROLLED_GFX) X(UNCONTROLLED_MEM) X(ALIGNMENT_UNVERIFIED) X(RAIL_SOURCE_CHANGED) \
  X(PEAK_GRAPHICS_PROXY) X(PEAK_UNAVAILABLE) X(STATE_MISMATCH) X(CAP_MISMATCH) X(CLOCK_MISMATCH) X(TEMP_MISMATCH)

#define PM_ENUM_PO(name) PM_PO_##name,
#define PM_ENUM_PF(name) PM_PF_##name,
#define PM_ENUM_TO(name) PM_TO_##name,
#define PM_ENUM_IT(name) PM_IT_##name,
#define PM_ENUM_IB(name) PM_IB_##name,
#define PM_ENUM_IP(name) PM_IP_##name,
#define PM_ENUM_W(name) PM_W_##name,

enum { PM_PHASE_FIELDS(PM_ENUM_PO) PM_PO_COUNT };
enum { PM_PHASE_FLAGS(PM_ENUM_PF) PM_PF_COUNT };
enum { PM_TRIAL_FIELDS(PM_ENUM_TO) PM_TO_COUNT };
enum { PM_ISSUES_TREATMENT(PM_ENUM_IT) PM_IT_COUNT };
enum { PM_ISSUES_BASELINE(PM_ENUM_IB) PM_IB_COUNT };
enum { PM_ISSUES_PAIRED(PM_ENUM_IP) PM_IP_COUNT };
enum { PM_WARNINGS(PM_ENUM_W) PM_W_COUNT };

enum { PM_ISSUE_WORDS = 4, PM_N_METRICS = 47 };
static_assert(PM_PF_COUNT <= 32, "phase flags fit a 32-bit word");
static_assert(PM_IT_COUNT <= 64 && PM_IB_COUNT <= 64 && PM_IP_COUNT <= 64 && PM_W_COUNT <= 64, "issue words");

// The reference's _METRICS tuple (analysis.py:1059-1074), in order.
#define PM_METRIC_NAMES(X) \
  X(board_power_w) X(idle_power_w) X(incremental_power_w) X(throughput_ops_s) X(throughput_bytes_s) \
  X(pj_per_op) X(pj_per_logical_byte) X(total_pj_per_op) X(total_pj_per_logical_byte) \
  X(memory_rail_power_w) X(memory_rail_incremental_power_w) X(graphics_clock_mhz) X(sm_clock_mhz) X(memory_clock_mhz) \
  X(temperature_c) X(idle_fraction_of_measured_power) X(idle_fraction_of_power_limit) X(power_limit_utilization) \
  X(tensor_peak_tflops_at_achieved_clock) X(tensor_utilization_vs_dense_clock_peak) \
  X(total_pj_per_flop) X(total_pj_per_logical_bit) \
  X(operational_idle_increment_power_w) X(operational_idle_increment_energy_j) \
  X(operational_idle_increment_pj_per_flop) X(operational_idle_increment_pj_per_logical_bit) \
  X(paired_active_reference_power_w) X(paired_active_reference_energy_j) \
  X(paired_active_reference_pj_per_flop) X(paired_active_reference_pj_per_logical_bit) \
  X(throughput_elements_s) X(throughput_rows_s) X(total_pj_per_element) X(total_pj_per_row) \
  X(operational_idle_increment_pj_per_element) X(operational_idle_increment_pj_per_row) \
  X(paired_active_reference_pj_per_element) X(paired_active_reference_pj_per_row) \
  X(throughput_sfu_instructions_s) X(total_pj_per_instruction) X(operational_idle_increment_pj_per_instruction) \
  X(paired_active_reference_pj_per_instruction) X(sfu_reference_delta_pj_per_instruction) X(sfu_reference_delta_power_w) \
  X(active_reference_duration_s) X(active_reference_counted_loop_slots) X(active_reference_loop_slots_s)
#define PM_ENUM_M(name) PM_M_##name,
enum { PM_METRIC_NAMES(PM_ENUM_M) PM_M_COUNT };
static_assert((int)PM_M_COUNT == (int)PM_N_METRICS, "the reference's _METRICS has 47 entries");
