// powerbench-compatible workload engine: argv grammar, device record, phased
// run loop with completion epochs, post-run checks and JSONL records.
//
// The command line, the phase order (warmup -> idle_pre -> [warmup_reference
// -> active_reference] <-> [warmup_treatment -> measure] -> idle_post), the
// epoch rule (about one second, closed after a completed batch, admission
// counters read back inside the window) and the record fields are the
// contract that powermodeling's runner and analysis consume
// (cuda/gpu_bench.cu:121-254, 519-602, 820-1174; cuda/sfu.cuh:226-356 in the
// reference); the kernels behind them are libpmb200's own (workloads.cu,
// tensor.cu).  Lines go to a caller callback; pm_powerbench returns 0, or 1
// with the error text in pm_last_error (the executable prints it to stderr as
// "powerbench: <msg>").
#include <cublas_v2.h>
#include <cuda_profiler_api.h>
#include <cuda_runtime.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <limits>
#include <numeric>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "pmb200.h"
#include "pm_capi.h"
#include "tensor.cuh"
#include "workloads.cuh"

namespace pm {
namespace {

struct Failure : std::runtime_error { using std::runtime_error::runtime_error; };

void check(cudaError_t e, const char* where) {
  if (e != cudaSuccess) throw Failure(std::string(where) + ": " + cudaGetErrorString(e));
}
void check_blas(cublasStatus_t e, const char* where) {
  if (e != CUBLAS_STATUS_SUCCESS) throw Failure(std::string(where) + ": cuBLAS status " + std::to_string(int(e)));
}

uint64_t monotonic_ns() {
  timespec ts{};
  if (clock_gettime(CLOCK_MONOTONIC, &ts) != 0) throw Failure("clock_gettime(CLOCK_MONOTONIC) failed");
  return uint64_t(ts.tv_sec) * 1000000000ULL + uint64_t(ts.tv_nsec);
}

// ---------------------------------------------------------------- JSON lines
std::string quoted(const std::string& v) {
  std::string out = "\"";
  for (unsigned char c : v) {
    if (c == '"' || c == '\\') { out += '\\'; out += char(c); }
    else if (c < 32) { char buf[8]; snprintf(buf, sizeof buf, "\\u%04x", c); out += buf; }
    else out += char(c);
  }
  return out + "\"";
}
std::string num(double v) {
  if (!std::isfinite(v)) return "null";
  char buf[40];
  snprintf(buf, sizeof buf, "%.17g", v);
  return buf;
}

class Obj {
 public:
  Obj& raw(const char* k, const std::string& v) { sep(); s_ += quoted(k) + ":" + v; return *this; }
  Obj& str(const char* k, const std::string& v) { return raw(k, quoted(v)); }
  Obj& f(const char* k, double v) { return raw(k, num(v)); }
  Obj& u(const char* k, uint64_t v) { return raw(k, std::to_string(v)); }
  Obj& i(const char* k, long long v) { return raw(k, std::to_string(v)); }
  Obj& b(const char* k, bool v) { return raw(k, v ? "true" : "false"); }
  Obj& null(const char* k) { return raw(k, "null"); }
  Obj& opt_str(const char* k, bool present, const std::string& v) { return present ? str(k, v) : null(k); }
  std::string done() const { return "{" + s_ + "}"; }
 private:
  void sep() { if (!s_.empty()) s_ += ","; }
  std::string s_;
};

struct Sink {
  pm_line_cb cb;
  void* user;
  void line(const std::string& s) const { cb(s.c_str(), user); }
};

void phase_line(const Sink& out, const char* name, const char* event) {
  out.line(Obj().str("type", "phase").str("phase", name).str("event", event).u("host_monotonic_ns", monotonic_ns()).done());
}

// ---------------------------------------------------------------- options
bool is_sfu(const std::string& w) {
  return w == "sfu_ex2" || w == "sfu_lg2" || w == "sfu_rcp" || w == "sfu_rsqrt" || w == "sfu_sqrt" || w == "sfu_tanh";
}
bool is_nonlinear(const std::string& w) {
  return w == "exp" || w == "tanh" || w == "silu" || w == "rmsnorm" || w == "softmax";
}

struct Options {
  int device = 0, blocks = 0, threads = 256, accumulators = 4;
  int gemm_m = 4096, gemm_n = 4096, gemm_k = 4096;
  double seconds = 10, warmup_seconds = 3, idle_seconds = 6;
  uint64_t working_set_bytes = 0, stride = 1, iterations = 0;
  int batch_launches = 0;
  uint64_t fixed_batches = 0, warmup_batches = 0, offset_bytes = 0, seed = 1;
  std::string workload = "tensor", access = "read", reference_order = "AB", read_cache_policy = "auto", grid_mode = "auto";
  uint64_t sfu_lanes = 262144;
  int sfu_chains = 4;
  int vector_bytes = 4;            // 4: scalar reference access; 16: one uint4 per access
  std::string chase_granularity = "word";
  std::string nonlinear_mode;      // "streaming" opts in to the complete nonlinear functions
  int row_width = 0;               // RMSNorm/softmax row width (default 1024)
  bool nonlinear_mode_explicit = false;
  bool tensor_uniform = false;     // fp16 operands uniform[-1,1) instead of [-0.25,0.25)
  int fill = FILL_RANDOM_WORD;     // memory payload: random_word (the reference's) or a seeded uint32 LCG
  int sfu_input = SFU_INPUT_PARITY;  // SFU operands: the reference's [0.5,1) or uniform [0.5,2) with XOR checksums
  std::vector<unsigned> sm_ids;
  bool describe = false, profile_region = false, paired_reference = false;
  bool blocks_explicit = false, grid_mode_explicit = false, sfu_explicit = false;
  bool policy_explicit = false, stride_elements_flag = false, stride_words_flag = false;
};

uint64_t parse_u64(const std::string& v, const char* flag) {
  if (v.empty() || v[0] == '-') throw Failure(std::string(flag) + " requires an unsigned integer");
  size_t used = 0;
  uint64_t out = 0;
  try { out = std::stoull(v, &used, 10); } catch (...) { throw Failure(std::string(flag) + " requires an integer"); }
  if (used != v.size()) throw Failure(std::string(flag) + " requires an integer");
  return out;
}
int parse_int(const std::string& v, const char* flag) {
  const uint64_t x = parse_u64(v, flag);
  if (x > uint64_t(std::numeric_limits<int>::max())) throw Failure(std::string(flag) + " is too large");
  return int(x);
}
double parse_seconds(const std::string& v, const char* flag) {
  size_t used = 0;
  double x = 0;
  try { x = std::stod(v, &used); } catch (...) { used = 0; }
  if (used != v.size() || !std::isfinite(x) || x < 0) throw Failure(std::string(flag) + " requires a finite nonnegative number");
  return x;
}

const char* kUsage =
  "powerbench --describe [--device N]\n"
  "powerbench --workload tensor|gemm|l1|l2|l2_latency|hbm|control|sfu_ex2|sfu_lg2|sfu_rcp|sfu_rsqrt|sfu_sqrt|sfu_tanh [options]\n"
  "powerbench --workload exp|tanh|silu|rmsnorm|softmax --nonlinear-mode streaming [--row-width 1024] [options]\n"
  "  --device N --seconds 10 --warmup-seconds 3 --idle-seconds 6\n"
  "  --blocks N --threads 256 --iterations N --tensor-accumulators 1..8\n"
  "  --batch-launches N --fixed-batches N --warmup-batches N --profile-region\n"
  "  --paired-reference --reference-order AB|BA\n"
  "  --working-set-bytes N --stride-words N (alias --stride-elements) --offset-bytes N\n"
  "  --access read|write|copy --sm-ids 0,1,... --seed N --read-cache-policy auto|ca|cg|cs\n"
  "  --gemm-m 4096 --gemm-n 4096 --gemm-k 4096 --grid-mode auto|fixed (nonlinear/SFU) --sfu-lanes N --sfu-chains 1|4|8\n"
  "  --nonlinear-mode streaming (required opt-in for complete exp/tanh/silu/rmsnorm/softmax)\n"
  "  --row-width N (RMSNorm/softmax row width, 1..65536, default 1024)\n"
  "  --memory-vector-bytes 4|16 (16: one 16-byte access per thread and iteration)\n"
  "  --chase-granularity word|line (line: 64-bit links on 128-byte lines)\n"
  "  --tensor-input uniform (fp16 operands uniform in [-1,1))\n"
  "  --fill random_word|lcg (memory payload; lcg: seeded uint32 LCG 1664525 x + 1013904223)\n"
  "  --sfu-input reference|uniform_0p5_2 (uniform_0p5_2: thread-hash operands in [0.5,2), per-thread XOR checksum)\n"
  "stdout is JSONL, except for this --help text.\n";

Options parse_options(int argc, const char* const* argv, const Sink& out, bool* help) {
  Options o;
  *help = false;
  for (int k = 1; k < argc; ++k) {
    const std::string flag = argv[k];
    if (flag == "--help" || flag == "-h") { *help = true; return o; }
    if (flag == "--describe") { o.describe = true; continue; }
    if (flag == "--profile-region") { o.profile_region = true; continue; }
    if (flag == "--paired-reference") { o.paired_reference = true; continue; }
    if (k + 1 >= argc) throw Failure("missing value for " + flag);
    const std::string v = argv[++k];
    const char* f = flag.c_str();
    if (flag == "--device") o.device = parse_int(v, f);
    else if (flag == "--blocks") { o.blocks = parse_int(v, f); o.blocks_explicit = true; }
    else if (flag == "--threads") o.threads = parse_int(v, f);
    else if (flag == "--grid-mode") { o.grid_mode = v; o.grid_mode_explicit = true; }
    else if (flag == "--sfu-lanes") { o.sfu_lanes = parse_u64(v, f); o.sfu_explicit = true; }
    else if (flag == "--sfu-chains") { o.sfu_chains = parse_int(v, f); o.sfu_explicit = true; }
    else if (flag == "--batch-launches") o.batch_launches = parse_int(v, f);
    else if (flag == "--fixed-batches") o.fixed_batches = parse_u64(v, f);
    else if (flag == "--warmup-batches") o.warmup_batches = parse_u64(v, f);
    else if (flag == "--seconds") o.seconds = parse_seconds(v, f);
    else if (flag == "--warmup-seconds") o.warmup_seconds = parse_seconds(v, f);
    else if (flag == "--idle-seconds") o.idle_seconds = parse_seconds(v, f);
    else if (flag == "--iterations") o.iterations = parse_u64(v, f);
    else if (flag == "--working-set-bytes") o.working_set_bytes = parse_u64(v, f);
    else if (flag == "--stride-elements") { o.stride = parse_u64(v, f); o.stride_elements_flag = true; }
    else if (flag == "--stride-words") { o.stride = parse_u64(v, f); o.stride_words_flag = true; }
    else if (flag == "--offset-bytes") o.offset_bytes = parse_u64(v, f);
    else if (flag == "--seed") o.seed = parse_u64(v, f);
    else if (flag == "--tensor-accumulators") o.accumulators = parse_int(v, f);
    else if (flag == "--reference-order") o.reference_order = v;
    else if (flag == "--workload") o.workload = v;
    else if (flag == "--access") o.access = v;
    else if (flag == "--read-cache-policy") { o.read_cache_policy = v; o.policy_explicit = true; }
    else if (flag == "--gemm-m") o.gemm_m = parse_int(v, f);
    else if (flag == "--gemm-n") o.gemm_n = parse_int(v, f);
    else if (flag == "--gemm-k") o.gemm_k = parse_int(v, f);
    else if (flag == "--memory-vector-bytes") o.vector_bytes = parse_int(v, f);
    else if (flag == "--chase-granularity") o.chase_granularity = v;
    else if (flag == "--fill") {
      if (v != "random_word" && v != "lcg") throw Failure("--fill must be random_word or lcg");
      o.fill = v == "lcg" ? FILL_LCG : FILL_RANDOM_WORD;
    }
    else if (flag == "--sfu-input") {
      if (v != "reference" && v != "uniform_0p5_2") throw Failure("--sfu-input must be reference or uniform_0p5_2");
      o.sfu_input = v == "uniform_0p5_2" ? SFU_INPUT_UNIFORM_0P5_2 : SFU_INPUT_PARITY;
      o.sfu_explicit = true;
    }
    else if (flag == "--tensor-input") { if (v != "uniform" && v != "reference") throw Failure("--tensor-input must be uniform or reference"); o.tensor_uniform = v == "uniform"; }
    else if (flag == "--nonlinear-mode") { o.nonlinear_mode = v; o.nonlinear_mode_explicit = true; }
    else if (flag == "--row-width") {
      o.row_width = parse_int(v, f);
      if (!o.row_width) throw Failure("--row-width must be positive");
    }
    else if (flag == "--sm-ids") {
      std::stringstream ss(v);
      std::string item;
      while (std::getline(ss, item, ',')) {
        const uint64_t id = parse_u64(item, "--sm-ids");
        if (id >= kSmSlots) throw Failure("SM ID is outside supported telemetry range");
        o.sm_ids.push_back(unsigned(id));
      }
      if (o.sm_ids.empty()) throw Failure("--sm-ids cannot be empty");
      std::sort(o.sm_ids.begin(), o.sm_ids.end());
      o.sm_ids.erase(std::unique(o.sm_ids.begin(), o.sm_ids.end()), o.sm_ids.end());
    } else throw Failure("unknown option " + flag);
  }
  (void)out;
  // Guards of the reference's grammar (gpu_bench.cu:200-254).
  const bool memory = o.workload == "l1" || o.workload == "l2" || o.workload == "hbm";
  if (o.seconds <= 0) throw Failure("--seconds must be positive");
  const bool cache_read = o.access == "read" && memory;
  if (o.read_cache_policy != "auto" && o.read_cache_policy != "ca" && o.read_cache_policy != "cg" && o.read_cache_policy != "cs")
    throw Failure("--read-cache-policy must be auto, ca, cg or cs");
  if (o.policy_explicit && !cache_read) throw Failure("--read-cache-policy applies only to L1/L2/HBM read workloads");
  if (cache_read) {
    if (o.read_cache_policy == "auto") o.read_cache_policy = o.workload == "l1" ? "ca" : "cg";
    if ((o.workload == "l1" && o.read_cache_policy != "ca") || (o.workload == "l2" && o.read_cache_policy != "cg"))
      throw Failure("--read-cache-policy requires ca for L1 and cg for L2; HBM supports ca/cg/cs");
  }
  if (o.reference_order != "AB" && o.reference_order != "BA") throw Failure("--reference-order must be AB or BA");
  if (o.paired_reference && !o.profile_region && o.workload != "control" && (o.seconds < 10 || o.warmup_seconds < 1 || o.idle_seconds < 6))
    throw Failure("paired energy arms require seconds>=10, warmup-seconds>=1 and idle-seconds>=6");
  if (o.stride_elements_flag && o.stride_words_flag)
    throw Failure("choose only one of --stride-words and --stride-elements; both flags use 32-bit word units");
  if (o.stride == 0 || o.stride > (1ULL << 32)) throw Failure("invalid --stride-words/--stride-elements");
  if (o.accumulators < 1 || o.accumulators > 8) throw Failure("--tensor-accumulators must be 1..8");
  if (o.threads < 32 || o.threads > 1024 || o.threads % 32) throw Failure("--threads must be a multiple of 32 between 32 and 1024");
  if (o.offset_bytes % 4 || o.working_set_bytes % 4) throw Failure("memory offset/footprint must be multiples of 4 bytes");
  if (o.iterations > (1ULL << 32)) throw Failure("--iterations must be <= 2^32");
  if (o.batch_launches > 65536) throw Failure("--batch-launches must be <= 65536");
  const bool nonlinear = is_nonlinear(o.workload);
  const bool known = o.workload == "tensor" || o.workload == "gemm" || memory || o.workload == "l2_latency" || o.workload == "control" ||
                     is_sfu(o.workload) || nonlinear;
  if (!known) throw Failure("unknown workload " + o.workload);
  if (nonlinear && o.nonlinear_mode != "streaming")
    throw Failure("complete nonlinear functions require explicit --nonlinear-mode streaming; these include global I/O and supporting arithmetic/reductions; use sfu_* workloads for SFU-only experiments (EXP is not EX2)");
  if (!nonlinear && o.nonlinear_mode_explicit)
    throw Failure("--nonlinear-mode streaming applies only to complete exp/tanh/silu/rmsnorm/softmax workloads");
  if (o.access != "read" && o.access != "write" && o.access != "copy") throw Failure("unknown memory access " + o.access);
  if (o.workload == "l1" && o.access != "read") throw Failure("L1 global-store/copy attribution is unsupported; use L1 read");
  if (o.workload == "l2_latency" && o.access != "read") throw Failure("dependent latency probes support read only");
  if (o.workload == "l2_latency" && o.stride != 1) throw Failure("latency probes use randomized dependent links; --stride-elements must be 1");
  if (o.workload == "gemm" && !o.sm_ids.empty()) throw Failure("cuBLAS GEMM cannot honor --sm-ids");
  if (o.gemm_m <= 0 || o.gemm_n <= 0 || o.gemm_k <= 0) throw Failure("GEMM dimensions must be positive");
  const bool rowwise = o.workload == "rmsnorm" || o.workload == "softmax";
  if (rowwise && !o.row_width) o.row_width = 1024;
  if ((rowwise && o.row_width > 65536) || (!rowwise && o.row_width))
    throw Failure("--row-width 1..65536 applies only to RMSNorm/Softmax");
  if (nonlinear && (!o.sm_ids.empty() || o.offset_bytes || o.stride != 1 || o.access != "read"))
    throw Failure("nonlinear workloads require a full grid, offset=0, stride=1 and access=read");
  if (o.grid_mode != "auto" && o.grid_mode != "fixed") throw Failure("--grid-mode must be auto or fixed");
  if (o.grid_mode_explicit && !is_sfu(o.workload) && !nonlinear) throw Failure("--grid-mode applies only to nonlinear/SFU workloads");
  if ((is_sfu(o.workload) || nonlinear) && o.grid_mode == "fixed" && (!o.blocks_explicit || o.blocks <= 0))
    throw Failure("fixed nonlinear/SFU grid requires explicit positive --blocks");
  if (!o.sfu_lanes || (o.sfu_chains != 1 && o.sfu_chains != 4 && o.sfu_chains != 8))
    throw Failure("--sfu-lanes must be positive and --sfu-chains must be 1, 4 or 8");
  if (o.sfu_explicit && !is_sfu(o.workload)) throw Failure("--sfu-lanes/--sfu-chains apply only to register SFU workloads");
  if (is_sfu(o.workload) && (!o.sm_ids.empty() || o.working_set_bytes || o.offset_bytes || o.stride != 1 || o.access != "read"))
    throw Failure("register SFU uses --sfu-lanes, no global input buffer, SM filter, offset, stride or memory access mode");
  if (o.vector_bytes != 4 && o.vector_bytes != 16) throw Failure("--memory-vector-bytes must be 4 or 16");
  if (o.vector_bytes == 16 && (!(o.workload == "hbm" || o.workload == "l2") || o.access == "write"))
    throw Failure("--memory-vector-bytes 16 applies to L2/HBM read and copy");
  if (o.vector_bytes == 16 && o.offset_bytes % 16) throw Failure("16-byte accesses need --offset-bytes to be a multiple of 16");
  if (o.fill == FILL_LCG && o.workload != "l1" && o.workload != "l2" && o.workload != "hbm")
    throw Failure("--fill applies only to l1/l2/hbm memory workloads");
  if (o.chase_granularity != "word" && o.chase_granularity != "line") throw Failure("--chase-granularity must be word or line");
  if (o.chase_granularity == "line" && o.workload != "l2_latency") throw Failure("--chase-granularity applies only to l2_latency");
  return o;
}

// ---------------------------------------------------------------- device record
template <class T> struct DevBuf {
  T* p = nullptr;
  explicit DevBuf(size_t n) { check(cudaMalloc(reinterpret_cast<void**>(&p), std::max<size_t>(1, n) * sizeof(T)), "cudaMalloc"); }
  ~DevBuf() { if (p) cudaFree(p); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
};

std::string uuid_text(const cudaUUID_t& u) {
  char buf[64];
  const unsigned char* b = reinterpret_cast<const unsigned char*>(u.bytes);
  snprintf(buf, sizeof buf, "GPU-%02x%02x%02x%02x-%02x%02x-%02x%02x-%02x%02x-%02x%02x%02x%02x%02x%02x",
           b[0], b[1], b[2], b[3], b[4], b[5], b[6], b[7], b[8], b[9], b[10], b[11], b[12], b[13], b[14], b[15]);
  return buf;
}

void describe(const Options& o, const cudaDeviceProp& p, const Sink& out) {
  char pci[64] = {};
  check(cudaDeviceGetPCIBusId(pci, sizeof pci, o.device), "cudaDeviceGetPCIBusId");
  int runtime = 0, driver = 0, blas = 0, max_blocks = 0, sm_khz = 0, mem_khz = 0;
  { cublasHandle_t h; check_blas(cublasCreate(&h), "cublasCreate"); cublasGetVersion(h, &blas); cublasDestroy(h); }
  check(cudaRuntimeGetVersion(&runtime), "cudaRuntimeGetVersion");
  check(cudaDriverGetVersion(&driver), "cudaDriverGetVersion");
  check(cudaDeviceGetAttribute(&max_blocks, cudaDevAttrMaxBlocksPerMultiprocessor, o.device), "attr");
  check(cudaDeviceGetAttribute(&sm_khz, cudaDevAttrClockRate, o.device), "attr");
  check(cudaDeviceGetAttribute(&mem_khz, cudaDevAttrMemoryClockRate, o.device), "attr");
  out.line(Obj().str("type", "device").i("process_id", getpid()).i("cuda_ordinal", o.device).str("name", p.name)
               .str("uuid", uuid_text(p.uuid)).str("pci_bus_id", pci)
               .str("cc", std::to_string(p.major) + "." + std::to_string(p.minor))
               .i("compute_capability_major", p.major).i("compute_capability_minor", p.minor)
               .i("sm_count", p.multiProcessorCount).i("warp_size", p.warpSize).u("l2_bytes", p.l2CacheSize)
               .u("total_memory_bytes", p.totalGlobalMem).i("max_threads_per_sm", p.maxThreadsPerMultiProcessor)
               .i("max_blocks_per_sm", max_blocks).i("registers_per_sm", p.regsPerMultiprocessor)
               .u("shared_memory_per_sm_bytes", p.sharedMemPerMultiprocessor)
               .i("nominal_max_sm_clock_khz", sm_khz).i("nominal_max_memory_clock_khz", mem_khz)
               .i("memory_bus_width_bits", p.memoryBusWidth).i("cuda_runtime_version", runtime)
               .i("cuda_driver_version", driver).i("cuda_compile_version", CUDART_VERSION).i("cublas_version", blas)
               .str("implementation", "libpmb200 sm_100a").done());
}

// ---------------------------------------------------------------- phase engine
struct Epoch { uint64_t start_ns = 0, end_ns = 0, batches = 0, admitted = 0, readback_ns = 0; };
struct Timing { double device_s = 0, host_s = 0; uint64_t batches = 0; std::vector<Epoch> epochs; };

struct Event {
  cudaEvent_t e{};
  Event() { check(cudaEventCreate(&e), "cudaEventCreate"); }
  ~Event() { cudaEventDestroy(e); }
};

Timing run_phase(const Sink& out, const char* name, double seconds, uint64_t fixed_batches, const std::function<void()>& launch,
                 const std::function<uint64_t()>& snapshot = {}, bool profile_region = false) {
  check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  phase_line(out, name, "start");
  Event start, stop, batch_done;
  if (profile_region) check(cudaProfilerStart(), "cudaProfilerStart");
  const uint64_t begin = monotonic_ns();
  check(cudaEventRecord(start.e), "cudaEventRecord");
  uint64_t batches = 0, epoch_begin = begin, epoch_batches = 0, previous = 0;
  Timing t;
  auto close_epoch = [&] {
    const uint64_t copy_begin = monotonic_ns();
    const uint64_t cumulative = snapshot ? snapshot() : 0;
    const uint64_t copy_end = monotonic_ns();
    t.epochs.push_back({epoch_begin, copy_end, batches - epoch_batches, cumulative - previous, copy_end - copy_begin});
    epoch_begin = copy_end; epoch_batches = batches; previous = cumulative;
  };
  while (fixed_batches ? batches < fixed_batches
                       : (batches == 0 ? seconds > 0 : double(monotonic_ns() - begin) * 1e-9 < seconds)) {
    launch();
    check(cudaGetLastError(), "kernel launch");
    check(cudaEventRecord(batch_done.e), "cudaEventRecord");
    check(cudaEventSynchronize(batch_done.e), "kernel batch");
    ++batches;
    if (snapshot && monotonic_ns() - epoch_begin >= 1000000000ULL) close_epoch();
  }
  check(cudaEventRecord(stop.e), "cudaEventRecord");
  check(cudaEventSynchronize(stop.e), "cudaEventSynchronize");
  if (snapshot && batches > epoch_batches) close_epoch();
  const uint64_t end = monotonic_ns();
  if (profile_region) check(cudaProfilerStop(), "cudaProfilerStop");
  float ms = 0;
  check(cudaEventElapsedTime(&ms, start.e, stop.e), "cudaEventElapsedTime");
  phase_line(out, name, "end");
  t.device_s = double(ms) * 1e-3;
  t.host_s = double(end - begin) * 1e-9;
  t.batches = batches;
  return t;
}

void idle_phase(const Sink& out, const char* name, double seconds) {
  check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  phase_line(out, name, "start");
  std::this_thread::sleep_for(std::chrono::duration<double>(seconds));
  phase_line(out, name, "end");
}

std::string epochs_json(const Timing& t, int batch_launches, const std::function<void(Obj&, const Epoch&)>& counts) {
  std::string s = "[";
  for (size_t k = 0; k < t.epochs.size(); ++k) {
    const Epoch& e = t.epochs[k];
    Obj o;
    o.u("host_monotonic_start_ns", e.start_ns).u("host_monotonic_end_ns", e.end_ns)
     .f("start_s", double(e.start_ns) * 1e-9).f("end_s", double(e.end_ns) * 1e-9)
     .u("batches", e.batches).u("admitted_blocks", e.admitted).u("kernel_launches", e.batches * uint64_t(batch_launches));
    counts(o, e);
    o.b("counts_exact", true).u("counter_readback_ns", e.readback_ns);
    s += (k ? "," : "") + o.done();
  }
  return s + "]";
}

std::string resources_json(const cudaFuncAttributes& a, int max_blocks, int threads, const cudaDeviceProp& p, int blocks,
                           size_t dynamic_smem = 0) {
  return Obj().i("registers_per_thread", a.numRegs).u("local_bytes_per_thread", a.localSizeBytes)
      .u("static_shared_bytes_per_block", a.sharedSizeBytes).u("dynamic_shared_bytes_per_block", dynamic_smem)
      .i("max_active_blocks_per_sm", max_blocks).i("max_active_warps_per_sm", max_blocks * (threads / p.warpSize))
      .f("occupancy_upper_bound_fraction", double(max_blocks * threads) / p.maxThreadsPerMultiProcessor)
      .f("grid_average_blocks_per_sm", double(blocks) / p.multiProcessorCount)
      .str("scope", "compiled resources and theoretical residency bound; not achieved occupancy").done();
}

std::string protocol_json(const Options& o, bool paired, bool context, bool geometry_matched, const char* reference_kind,
                          const char* scope) {
  return Obj().str("type", "treatment_protocol").str("kind", paired ? "paired_active_reference" : "powered_idle_bracket")
      .raw("order", paired ? quoted(o.reference_order) : "null")
      .raw("phase_order", paired ? (o.reference_order == "AB" ? "[\"active_reference\",\"measure\"]" : "[\"measure\",\"active_reference\"]") : "[\"measure\"]")
      .b("same_process", true).b("same_allocations", true).b("same_clock_policy", true)
      .b("paired_reference_context_allocated", context).b("launch_geometry_matched", paired && geometry_matched)
      .raw("reference_workload", paired ? "\"control\"" : "null")
      .raw("reference_kind", paired ? quoted(reference_kind) : "null")
      .u("reference_iterations", paired ? o.iterations : 0).f("arm_seconds", o.seconds)
      .f("arm_warmup_seconds", o.warmup_seconds).str("reference_scope", scope).done();
}

uint64_t checksum_words(const std::vector<uint32_t>& v) {
  uint64_t h = 0;
  for (uint32_t w : v) h = h * 1315423911ULL + w;
  return h;
}

// ---------------------------------------------------------------- SFU arm
int sfu_op(const std::string& w) {
  if (w == "sfu_ex2") return SFU_EX2;
  if (w == "sfu_tanh") return SFU_TANH;
  if (w == "sfu_rsqrt") return SFU_RSQRT;
  if (w == "sfu_rcp") return SFU_RCP;
  if (w == "sfu_lg2") return SFU_LG2;
  return SFU_SQRT;
}
const char* sfu_opcode(int op) {
  static const char* names[] = {"ex2.approx.ftz.f32", "tanh.approx.f32", "rsqrt.approx.ftz.f32",
                                "rcp.approx.ftz.f32", "lg2.approx.ftz.f32", "sqrt.approx.ftz.f32"};
  return names[op];
}

struct SfuCheck { uint64_t checked = 0; double max_abs = 0, max_rel = 0; bool passed = true; };

SfuCheck check_sfu(int op, uint32_t* sample, const Options& o) {
  check(launch_sfu_check(op, sample, o.sfu_lanes, o.seed, o.sfu_chains, 0, o.sfu_input), "sfu check launch");
  const float top = o.sfu_input == SFU_INPUT_UNIFORM_0P5_2 ? 2.0f : 1.0f;   // operands lie in [0.5, top)
  check(cudaDeviceSynchronize(), "sfu check");
  uint32_t host[16];
  check(cudaMemcpy(host, sample, sizeof host, cudaMemcpyDeviceToHost), "cudaMemcpy");
  SfuCheck r;
  for (int k = 0; k < 8; ++k) {
    float x, y;
    memcpy(&x, &host[2 * k], 4);
    memcpy(&y, &host[2 * k + 1], 4);
    const double dx = x;
    const double e = op == SFU_EX2 ? std::exp2(dx) : op == SFU_TANH ? std::tanh(dx) : op == SFU_RSQRT ? 1.0 / std::sqrt(dx)
                   : op == SFU_RCP ? 1.0 / dx : op == SFU_LG2 ? std::log2(dx) : std::sqrt(dx);
    const double err = std::fabs(double(y) - e), rel = err / std::max(std::fabs(e), 1e-30);
    r.max_abs = std::max(r.max_abs, err);
    r.max_rel = std::max(r.max_rel, rel);
    r.passed = r.passed && std::isfinite(x) && std::isfinite(y) && x >= 0.5f && x < top && err <= 2e-6 + 2e-5 * std::fabs(e);
    ++r.checked;
  }
  return r;
}

uint64_t sfu_checksum(const uint32_t* sink, uint64_t lanes) {
  const uint64_t count = std::min<uint64_t>(lanes, 64);
  uint64_t h = 0;
  for (uint64_t k = 0; k < count; ++k) {
    const uint64_t lane = count == 1 ? 0 : k * (lanes - 1) / (count - 1);
    uint32_t w = 0;
    check(cudaMemcpy(&w, sink + lane, 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
    h = h * 1315423911ULL + w;
  }
  return h;
}

// XOR of every lane's sink word (the BASELINE-mode per-thread XOR checksums folded into one).
uint32_t xor_all(const uint32_t* sink, uint64_t lanes) {
  std::vector<uint32_t> host(lanes);
  check(cudaMemcpy(host.data(), sink, lanes * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
  uint32_t x = 0;
  for (uint32_t w : host) x ^= w;
  return x;
}

void sfu_metadata(Obj& j, const Options& o, int op) {
  j.str("sfu_primitive", o.workload.substr(4)).u("sfu_lanes", o.sfu_lanes).i("sfu_chains", o.sfu_chains)
   .str("sfu_input_policy", o.sfu_input == SFU_INPUT_UNIFORM_0P5_2
                                ? "thread_hash_uniform_0p5_2_then_feedback_xor_iteration_mantissa_0p5_1_v1"
                                : "feedback_xor_iteration_mantissa_0p5_1_v1")
   .str("sfu_ptx_opcode", sfu_opcode(op))
   .b("sfu_approximate", true).b("sfu_flush_to_zero", op != SFU_TANH)
   .raw("sfu_exponent_base", (op == SFU_EX2 || op == SFU_LG2) ? "2" : "null")
   .str("math_implementation", "ptx_approx_register_v1").str("grid_mode", o.grid_mode)
   .str("block_completion_count_source", "synchronized_completed_launches");
}

void experiment_sfu(Options o, const cudaDeviceProp& p, const Sink& out) {
  const int op = sfu_op(o.workload);
  if (o.threads > p.maxThreadsPerBlock) throw Failure("register SFU requires supported threads");
  if (o.grid_mode == "auto") {
    const uint64_t blocks = o.sfu_lanes / o.threads + (o.sfu_lanes % o.threads != 0);
    if (blocks > 1000000 || blocks > uint64_t(p.maxGridSize[0]))
      throw Failure("SFU auto grid exceeds practical/hardware limit; choose an explicit fixed grid");
    if (o.blocks_explicit && uint64_t(o.blocks) != blocks)
      throw Failure("explicit --blocks must equal the SFU Q-derived auto grid; use --grid-mode fixed for a block sweep");
    o.blocks = int(blocks);
  }
  if (o.blocks <= 0 || o.blocks > 1000000 || o.blocks > p.maxGridSize[0]) throw Failure("SFU blocks exceed practical/hardware limit");
  if (!o.iterations) o.iterations = 16384;
  if (!o.batch_launches) o.batch_launches = 1;
  const bool context = o.paired_reference, paired = context && !o.profile_region;
  if ((long double)o.sfu_lanes * 4 * (context ? 2 : 1) + 262144 > (long double)p.totalGlobalMem * 0.7)
    throw Failure("SFU sink/context allocations exceed 70% of device memory");
  DevBuf<uint32_t> sink(o.sfu_lanes), ref_sink(context ? o.sfu_lanes : 1), sample(16);
  check(cudaMemset(sink.p, 0, o.sfu_lanes * 4), "cudaMemset");
  check(cudaMemset(ref_sink.p, 0, (context ? o.sfu_lanes : 1) * 4), "cudaMemset");
  cudaFuncAttributes ta{}, ca{};
  check(sfu_attributes(op, false, o.sfu_chains, &ta), "cudaFuncGetAttributes");
  check(sfu_attributes(op, true, o.sfu_chains, &ca), "cudaFuncGetAttributes");
  if (ta.localSizeBytes || ta.sharedSizeBytes || ca.localSizeBytes || ca.sharedSizeBytes)
    throw Failure("register SFU/control compiled with local/shared memory; reject spill-contaminated experiment");
  auto launch = [&](bool control) {
    for (int k = 0; k < o.batch_launches; ++k)
      check(launch_sfu(op, control, o.sfu_chains, control ? ref_sink.p : sink.p, o.sfu_lanes, o.iterations, o.seed,
                       o.blocks, o.threads, 0, o.sfu_input), "sfu launch");
  };
  SfuCheck numerical = check_sfu(op, sample.p, o);
  if (!numerical.passed) throw Failure("native SFU one-step output differs from CPU double reference");
  out.line(protocol_json(o, paired, context, true, "register_loop_without_sfu",
                         "same Q, chains, initialization, bit-remap, loop, hash epilogue, grid and batching; SFU primitive replaced by PTX MOV; board-power operational proxy, not an isolated SFU rail"));
  auto treat = [&] { launch(false); };
  auto ref = [&] { launch(true); };
  run_phase(out, "warmup", o.warmup_seconds, o.warmup_batches, treat);
  idle_phase(out, "idle_pre", o.idle_seconds);
  Timing t, rt;
  std::function<uint64_t()> none = [] { return uint64_t(0); };
  auto treatment_arm = [&] {
    if (paired) run_phase(out, "warmup_treatment", o.warmup_seconds, o.warmup_batches, treat);
    t = run_phase(out, "measure", o.seconds, o.fixed_batches, treat, none, o.profile_region);
  };
  auto reference_arm = [&] {
    run_phase(out, "warmup_reference", o.warmup_seconds, o.warmup_batches, ref);
    rt = run_phase(out, "active_reference", o.seconds, o.fixed_batches, ref, none);
  };
  if (paired && o.reference_order == "AB") reference_arm();
  treatment_arm();
  if (paired && o.reference_order == "BA") reference_arm();
  idle_phase(out, "idle_post", o.idle_seconds);
  // Completed CTAs follow from synchronized launches (no admission counters in the hot loop).
  for (Timing* tm : {&t, &rt})
    for (Epoch& e : tm->epochs) e.admitted = e.batches * uint64_t(o.batch_launches) * uint64_t(o.blocks);
  const SfuCheck post = check_sfu(op, sample.p, o);
  numerical.checked += post.checked;
  numerical.max_abs = std::max(numerical.max_abs, post.max_abs);
  numerical.max_rel = std::max(numerical.max_rel, post.max_rel);
  numerical.passed = numerical.passed && post.passed;
  const uint64_t checksum = sfu_checksum(sink.p, o.sfu_lanes);
  const uint64_t allocated = (o.sfu_lanes + (context ? o.sfu_lanes : 1) + 16) * 4;
  int tb = 0, cb = 0;
  check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&tb, sfu_kernel_handle(op, false, o.sfu_chains), o.threads, 0), "occupancy");
  check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&cb, sfu_kernel_handle(op, true, o.sfu_chains), o.threads, 0), "occupancy");
  auto arm = [&](const Timing& tm, bool control) {
    const uint64_t launches = tm.batches * uint64_t(o.batch_launches);
    const long double slots = (long double)launches * o.sfu_lanes * o.iterations * o.sfu_chains;
    Obj j;
    j.str("type", control ? "active_reference_result" : "result").str("workload", control ? "control" : o.workload)
     .str("access", "read").raw("reference_kind", control ? "\"register_loop_without_sfu\"" : "null")
     .str("kernel_implementation_version", control ? "sfu_register_control_v1" : "sfu_register_recurrence_v1");
    sfu_metadata(j, o, op);
    j.f("duration_s", tm.device_s).f("host_duration_s", tm.host_s).u("batches", tm.batches).i("batch_launches", o.batch_launches)
     .u("iterations_per_launch", o.iterations).u("iterations_per_batch", o.iterations * o.batch_launches)
     .u("kernel_launches", launches).u("workload_launches", launches).u("fixed_batches", o.fixed_batches)
     .u("warmup_batches", o.warmup_batches).f("mean_batch_duration_s", tm.device_s / double(std::max<uint64_t>(1, tm.batches)))
     .str("duration_scope", "CUDA event elapsed experiment window including gaps; not summed kernel busy time")
     .i("blocks", o.blocks).i("threads", o.threads).b("launch_geometry_applies", true).u("admitted_blocks", launches * o.blocks)
     .f("sfu_instructions", control ? 0.0 : double(slots)).f("reference_loop_slots", control ? double(slots) : 0.0)
     .f("operations", control ? 0.0 : double(slots)).u("logical_bytes", 0).u("elements", 0)
     .str("operation_unit", control ? "not target work; common register-loop slots" : "scalar-lane native SFU instructions; not FLOPs or complete-function elements")
     .f("throughput_ops_s", control ? 0.0 : double(slots) / tm.device_s).u("throughput_bytes_s", 0)
     .u("working_set_bytes", 0).u("requested_working_set_bytes", 0).u("allocated_bytes", allocated).u("seed", o.seed)
     .u("checksum", control ? sfu_checksum(ref_sink.p, o.sfu_lanes) : checksum)
     .str("checksum_kind", o.sfu_input == SFU_INPUT_UNIFORM_0P5_2 ? "distributed_per_lane_register_xor_sample"
                                                                  : "distributed_per_lane_register_fnv_hash_sample")
     .raw("sfu_thread_xor_checksum", o.sfu_input == SFU_INPUT_UNIFORM_0P5_2
                                         ? std::to_string(xor_all(control ? ref_sink.p : sink.p, o.sfu_lanes)) : "null")
     .raw("kernel_resources", resources_json(control ? ca : ta, control ? cb : tb, o.threads, p, o.blocks))
     .raw("control_kernel_resources", resources_json(ca, cb, o.threads, p, o.blocks))
     .raw("numerical_validation", Obj().u("checked_values", control ? 0 : numerical.checked)
                                      .f("max_absolute_error", control ? 0 : numerical.max_abs)
                                      .f("max_relative_error", control ? 0 : numerical.max_rel)
                                      .f("absolute_tolerance", 2e-6).f("relative_tolerance", 2e-5)
                                      .str("scope", "one-step native outputs at eight lanes vs CPU double before and after phases").done())
     .raw("sanity", Obj().b("finite_output_sample", control || numerical.passed)
                         .raw("numerical_validation_passed", control ? "null" : numerical.passed ? "true" : "false")
                         .b("requested_sm_coverage_complete", true).done())
     .b("profile_region", o.profile_region).b("paired_reference_context_allocated", context)
     .raw("active_sm_ids", "[]").raw("missing_requested_sm_ids", "[]").str("active_sm_distribution_status", "not_measured_register_sfu")
     .raw("measure_epochs", epochs_json(tm, o.batch_launches, [&](Obj& e, const Epoch& ep) {
        const uint64_t l = ep.batches * uint64_t(o.batch_launches);
        const double s = double((long double)l * o.sfu_lanes * o.iterations * o.sfu_chains);
        e.f("sfu_instructions", control ? 0.0 : s).f("reference_loop_slots", control ? s : 0.0)
         .f("operations", control ? 0.0 : s).u("logical_bytes", 0).u("elements", 0);
        sfu_metadata(e, o, op);
      }))
     .raw("auxiliary_work", Obj().f("logical_result_output_bytes", double((long double)launches * o.sfu_lanes * 4))
                                  .u("sm_admission_atomic_updates", 0).u("host_counter_readback_bytes", 0).done())
     .str("input_precision", "fp32").str("accumulator_precision", "uint32 feedback bits");
    return j.done();
  };
  if (paired) out.line(arm(rt, true));
  out.line(arm(t, false));
  if (!numerical.passed) throw Failure("native SFU one-step output failed CPU double validation after measurement");
}

// ---------------------------------------------------------------- nonlinear arms
int nonlinear_fn(const std::string& w) {
  return w == "exp" ? NL_EXP : w == "tanh" ? NL_TANH : w == "silu" ? NL_SILU : w == "softmax" ? NL_SOFTMAX : NL_RMSNORM;
}

struct NonlinearCheck { uint64_t checked = 0, checksum = 0; double max_abs = 0, max_rel = 0; bool passed = true; };

// Sampled CPU double check of the device outputs (nonlinear.cuh:97-143 rule):
// up to eight items (elements, or whole rows for softmax/RMSNorm) at the
// global first, middle, last and evenly spread positions; |y - e| <= 2e-6 +
// 2e-4 |e|; softmax rows must also sum to 1 within 2e-4.  The checksum folds
// the checked output bits in order (h = h * 1315423911 + bits).
NonlinearCheck check_nonlinear(const Options& o, int fn, const float* in, const float* outp, const float* gamma,
                               uint64_t q) {
  NonlinearCheck r;
  const bool rowwise = fn == NL_SOFTMAX || fn == NL_RMSNORM;
  const uint64_t width = rowwise ? uint64_t(o.row_width) : 1;
  const uint64_t items = q / width, samples = std::min<uint64_t>(items, 8);
  std::vector<float> weights(width, 1.0f), x(width), y(width);
  if (fn == NL_RMSNORM) check(cudaMemcpy(weights.data(), gamma, width * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
  auto compare = [&](float actual, double expected) {
    const double err = std::fabs(double(actual) - expected), rel = err / std::max(std::fabs(expected), 1e-30);
    r.max_abs = std::max(r.max_abs, err);
    r.max_rel = std::max(r.max_rel, rel);
    r.passed = r.passed && std::isfinite(actual) && std::isfinite(expected) && err <= 2e-6 + 2e-4 * std::fabs(expected);
    uint32_t bits;
    memcpy(&bits, &actual, 4);
    r.checksum = r.checksum * 1315423911ULL + bits;
    ++r.checked;
  };
  for (uint64_t k = 0; k < samples; ++k) {
    const uint64_t item = samples == 1 ? 0 : k == samples / 2 ? items / 2 : k * (items - 1) / (samples - 1);
    check(cudaMemcpy(x.data(), in + item * width, width * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
    check(cudaMemcpy(y.data(), outp + item * width, width * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
    if (!rowwise) {
      const double v = x[0];
      compare(y[0], fn == NL_EXP ? std::exp(v) : fn == NL_TANH ? std::tanh(v) : v / (1.0 + std::exp(-v)));
      continue;
    }
    const double maximum = *std::max_element(x.begin(), x.end());
    double sum = 0, ysum = 0;
    for (float v : x) sum += fn == NL_SOFTMAX ? std::exp(double(v) - maximum) : double(v) * v;
    for (uint64_t c = 0; c < width; ++c) {
      const double e = fn == NL_SOFTMAX ? std::exp(double(x[c]) - maximum) / sum
                                        : double(x[c]) / std::sqrt(sum / double(width) + double(1e-5f)) * weights[c];
      compare(y[c], e);
      ysum += y[c];
    }
    if (fn == NL_SOFTMAX) r.passed = r.passed && std::fabs(ysum - 1.0) <= 2e-4;
  }
  return r;
}

// The exp|tanh|silu|rmsnorm|softmax arms (gpu_bench.cu:611-631, 712-716,
// 796-818, 857-911, 930-933, 976-984, 1030-1176 for these workloads): Q =
// working-set bytes / 4 input elements; the auto grid is ceil(Q / threads)
// blocks (pointwise) or one block per row; completed CTAs and elements follow
// from synchronized launch counts (no per-CTA admission counters).
void experiment_nonlinear(Options o, const cudaDeviceProp& p, const Sink& out) {
  const int fn = nonlinear_fn(o.workload);
  const bool rowwise = fn == NL_SOFTMAX || fn == NL_RMSNORM;
  if (o.threads > p.maxThreadsPerBlock) throw Failure("thread count exceeds this device limit");
  if (!o.working_set_bytes) o.working_set_bytes = uint64_t(1048576) * 4;
  const uint64_t requested_ws = o.working_set_bytes;
  const uint64_t q = o.working_set_bytes / 4;
  if (!q || (rowwise && q % uint64_t(o.row_width)))
    throw Failure("nonlinear Q must be positive; rowwise Q must contain complete rows");
  if (o.grid_mode == "auto") {
    const uint64_t derived = rowwise ? q / uint64_t(o.row_width) : (q + o.threads - 1) / o.threads;
    if (derived > 1000000 || derived > uint64_t(p.maxGridSize[0]))
      throw Failure("nonlinear auto grid exceeds practical/hardware block limit; use explicit fixed grid for grid-stride traversal");
    if (o.blocks_explicit && uint64_t(o.blocks) != derived)
      throw Failure("explicit --blocks must equal the Q-derived auto grid; use --grid-mode fixed for a block sweep");
    o.blocks = int(derived);
  }
  if (o.blocks <= 0 || o.blocks > 1000000 || o.blocks > p.maxGridSize[0])
    throw Failure("--blocks must be positive within practical/hardware limit");
  if (!o.iterations) o.iterations = 1;
  if (!o.batch_launches) o.batch_launches = 16;
  const uint64_t lanes = uint64_t(o.blocks) * o.threads;
  const bool context = o.paired_reference, paired = context && !o.profile_region;
  const uint64_t gamma_count = fn == NL_RMSNORM ? uint64_t(o.row_width) : 1;
  if ((long double)q * 8 + gamma_count * 4 + 4 + (context ? lanes : 1) * 4 + 262144 > (long double)p.totalGlobalMem * 0.7)
    throw Failure("nonlinear input/output/gamma and reference allocations exceed 70% of device memory");
  const int width = rowwise ? o.row_width : 0;
  DevBuf<float> input(q), output(q), gamma(gamma_count);
  DevBuf<uint32_t> ref_sink(context ? lanes : 1);
  // Large-offset logits exercise max-subtracted softmax without overflow (gpu_bench.cu:712-716).
  check(launch_nonlinear_fill(input.p, q, o.seed, fn == NL_SOFTMAX ? 100.0f : 0.0f, 0, p.multiProcessorCount, 0), "fill");
  check(launch_nonlinear_fill(gamma.p, gamma_count, o.seed ^ 12345ULL, 0.0f, 1, p.multiProcessorCount, 0), "fill");
  check(cudaMemset(output.p, 0, q * 4), "cudaMemset");
  check(cudaMemset(ref_sink.p, 0, (context ? lanes : 1) * 4), "cudaMemset");
  check(cudaDeviceSynchronize(), "fill kernels");
  auto single = [&] {
    check(launch_nonlinear(fn, input.p, gamma.p, output.p, q, width, o.iterations, o.blocks, o.threads, 0), "nonlinear launch");
  };
  auto treat = [&] { for (int k = 0; k < o.batch_launches; ++k) single(); };
  auto ref = [&] {
    for (int k = 0; k < o.batch_launches; ++k)
      check(launch_control_plain(ref_sink.p, o.iterations, o.blocks, o.threads, 0), "control launch");
  };
  single();
  check(cudaDeviceSynchronize(), "nonlinear kernel");
  NonlinearCheck numerical = check_nonlinear(o, fn, input.p, output.p, gamma.p, q);
  if (!numerical.passed) throw Failure("nonlinear output differs from CPU double reference before measurement");
  const NonlinearLayout layout = nonlinear_layout(fn, q, width, o.blocks, o.threads);
  const size_t smem = layout.dynamic_smem;
  cudaFuncAttributes attr{};
  int max_blocks = 0;
  check(cudaFuncGetAttributes(&attr, layout.kernel), "cudaFuncGetAttributes");
  check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&max_blocks, layout.kernel, o.threads, smem), "occupancy");
  out.line(protocol_json(o, paired, context, true, "issue_loop",
                         "paired integer issue-loop operational contrast; launch geometry, iterations and batching match the nonlinear kernel; instruction mix, residency, register pressure, occupancy and duration per launch are not counterfactual equivalents; not isolated component energy"));
  run_phase(out, "warmup", o.warmup_seconds, o.warmup_batches, treat);
  idle_phase(out, "idle_pre", o.idle_seconds);
  Timing t, rt;
  std::function<uint64_t()> none = [] { return uint64_t(0); };
  auto treatment_arm = [&] {
    if (paired) run_phase(out, "warmup_treatment", o.warmup_seconds, o.warmup_batches, treat);
    t = run_phase(out, "measure", o.seconds, o.fixed_batches, treat, none, o.profile_region);
  };
  auto reference_arm = [&] {
    run_phase(out, "warmup_reference", o.warmup_seconds, o.warmup_batches, ref);
    rt = run_phase(out, "active_reference", o.seconds, o.fixed_batches, ref, none);
  };
  if (paired && o.reference_order == "AB") reference_arm();
  treatment_arm();
  if (paired && o.reference_order == "BA") reference_arm();
  idle_phase(out, "idle_post", o.idle_seconds);
  for (Timing* tm : {&t, &rt})
    for (Epoch& e : tm->epochs) { e.admitted = e.batches * uint64_t(o.batch_launches) * uint64_t(o.blocks); e.readback_ns = 0; }
  const NonlinearCheck post = check_nonlinear(o, fn, input.p, output.p, gamma.p, q);
  numerical.checked += post.checked;
  numerical.max_abs = std::max(numerical.max_abs, post.max_abs);
  numerical.max_rel = std::max(numerical.max_rel, post.max_rel);
  numerical.passed = numerical.passed && post.passed;
  const uint64_t bytes_per_element = rowwise ? 16 : 8;
  const std::string distribution = fn == NL_SOFTMAX ? "deterministic uniform FP32 [96,104); stable max subtraction"
                                                    : "deterministic uniform FP32 [-4,4)";
  const char* sm_scope = "no per-CTA SMID/admission telemetry; synchronized launch completion does not measure physical SM coverage";
  if (paired) {
    const uint64_t launches = rt.batches * uint64_t(o.batch_launches);
    Obj j;
    j.str("type", "active_reference_result").str("workload", "control").str("reference_kind", "issue_loop")
     .str("kernel_implementation_version", "integer_issue_loop_no_admission_v2")
     .str("block_completion_count_source", "synchronized_completed_launches")
     .str("active_sm_distribution_status", "not_measured_nonlinear").str("sm_distribution_scope", sm_scope)
     .f("duration_s", rt.device_s).f("host_duration_s", rt.host_s).u("batches", rt.batches).i("batch_launches", o.batch_launches)
     .u("iterations_per_launch", o.iterations).i("blocks", o.blocks).i("threads", o.threads)
     .u("admitted_blocks", launches * uint64_t(o.blocks)).u("operations", 0).u("logical_bytes", 0)
     .str("operation_unit", "not FLOPs or target bytes; integer issue-loop reference")
     .raw("measure_epochs", epochs_json(rt, o.batch_launches, [](Obj& e, const Epoch&) { e.u("operations", 0).u("logical_bytes", 0); }))
     .raw("sanity", Obj().b("requested_sm_coverage_complete", true).done())
     .str("scope", "active integer issue-loop reference measured in same CUDA process and allocated context; no target-operation normalization and no physical component attribution");
    out.line(j.done());
  }
  const uint64_t launches = t.batches * uint64_t(o.batch_launches);
  const long double elements = (long double)launches * q * o.iterations, bytes = elements * bytes_per_element;
  const bool finite = numerical.passed;
  Obj j;
  j.str("type", "result").str("workload", o.workload).str("access", "read")
   .f("duration_s", t.device_s).f("host_duration_s", t.host_s).u("batches", t.batches).u("iterations_per_launch", o.iterations)
   .u("iterations_per_batch", o.iterations * o.batch_launches).i("batch_launches", o.batch_launches)
   .u("workload_launches", launches).u("kernel_launches", launches).u("gemm_invocations", 0)
   .u("fixed_batches", o.fixed_batches).u("warmup_batches", o.warmup_batches)
   .f("mean_batch_duration_s", t.device_s / double(std::max<uint64_t>(1, t.batches)))
   .str("duration_scope", "CUDA event elapsed experiment window including gaps; not summed kernel busy time")
   .str("kernel_implementation_version", "fp32_complete_nonlinear_q_grid_v2")
   .str("nonlinear_mode", o.nonlinear_mode).str("grid_mode", o.grid_mode).u("input_elements", q)
   .f("elements_per_launch", double((long double)q * o.iterations))
   .str("block_completion_count_source", "synchronized_completed_launches")
   .raw("memory_accesses_per_thread_iteration", "null").raw("memory_read_checksum_scope", "null")
   .raw("read_cache_policy", "null").raw("memory_read_index_math", "null").raw("memory_read_validation", "null")
   .f("operations", double(elements))
   .str("operation_unit", "output elements of the complete function; not FLOPs or SFU instructions")
   .f("logical_bytes", double(bytes)).f("throughput_ops_s", double(elements) / t.device_s)
   .f("throughput_bytes_s", double(bytes) / t.device_s).i("blocks", o.blocks).i("threads", o.threads)
   .b("launch_geometry_applies", true).u("admitted_blocks", launches * uint64_t(o.blocks))
   .u("working_set_bytes", q * 4).u("requested_working_set_bytes", requested_ws)
   .raw("write_copy_thread_addresses_disjoint", "null")
   .u("allocated_bytes", (2 * q + gamma_count + (context ? lanes : 1)) * 4).u("l1_bytes_per_block", 0)
   .u("stride_elements", 1).u("offset_bytes", 0).raw("memory_word_bytes", "null").raw("stride_words", "null")
   .raw("lane_stride_bytes", "null").i("tensor_accumulators", o.accumulators)
   .i("gemm_m", o.gemm_m).i("gemm_n", o.gemm_n).i("gemm_k", o.gemm_k).u("seed", o.seed)
   .u("checksum", post.checksum).str("checksum_kind", "validated_fp32_nonlinear_output_sample_hash")
   .raw("kernel_resources", resources_json(attr, max_blocks, o.threads, p, o.blocks, smem))
   .i("row_width", rowwise ? o.row_width : 0).f("elements", double(elements))
   .f("row_evaluations", rowwise ? double(elements / o.row_width) : 0.0)
   .str("math_implementation", "cuda_fp32_q_grid_v2")
   .raw("rms_epsilon", fn == NL_RMSNORM ? "0.00001" : "null").b("affine_gamma", fn == NL_RMSNORM)
   .str("nonlinear_input_distribution", distribution)
   .str("nonlinear_scope", "complete FP32 function including global input/output and row reductions; repeated applications reload fixed input; no pure SFU or FLOP attribution")
   .raw("numerical_validation", Obj().u("checked_values", numerical.checked).f("max_absolute_error", numerical.max_abs)
                                     .f("max_relative_error", numerical.max_rel).f("absolute_tolerance", 2e-6)
                                     .f("relative_tolerance", 2e-4)
                                     .str("scope", "CPU double reference on global first/middle/last and distributed elements or complete rows before warmup and after measurement; includes pointwise tail; softmax row sums also checked; not exhaustive").done())
   .raw("sanity", Obj().b("finite_output_sample", finite).raw("memory_read_sample_matches_reference", "null")
                       .b("numerical_validation_passed", numerical.passed).b("requested_sm_coverage_complete", true).done())
   .b("profile_region", o.profile_region).b("paired_reference_context_allocated", context)
   .raw("measure_epochs", epochs_json(t, o.batch_launches, [&](Obj& e, const Epoch& ep) {
      const long double el = (long double)ep.batches * o.batch_launches * q * o.iterations;
      e.f("operations", double(el)).f("logical_bytes", double(el * bytes_per_element)).f("elements", double(el))
       .f("row_evaluations", rowwise ? double(el / o.row_width) : 0.0);
    }))
   .raw("auxiliary_work", Obj().u("logical_result_output_bytes", 0).u("sm_admission_atomic_updates", 0)
                                .u("host_counter_readback_bytes", 0).done())
   .str("epoch_scope", "approximately one second, exact synchronized completed batch counts; nonlinear work/completed CTAs derived from Q and launch geometry without per-CTA telemetry or counter readback; no interpolated partial-batch counts")
   .raw("active_sm_ids", "[]").str("active_sm_distribution_status", "not_measured_nonlinear")
   .str("sm_distribution_scope", sm_scope).raw("missing_requested_sm_ids", "[]")
   .str("cache_policy", "ld/st.global.cg; L1 bypass; L2/DRAM residency requires counters")
   .str("nonlinear_kernel_layout", layout.description)
   .str("sparsity", "dense").str("input_precision", "fp32").str("accumulator_precision", "fp32");
  out.line(j.done());
  if (!finite) throw Failure("non-finite or numerically incorrect output sample");
}

// ---------------------------------------------------------------- generic arms
// CPU oracle of the scalar read sum for sampled threads (gpu_bench.cu:937-973
// rule: repeated address cycles folded, at most 65536 unique steps per thread).
struct ReadCheck { uint64_t checked = 0, mismatched = 0; const char* status = "not_checked_iteration_budget"; };

ReadCheck check_read_sums(const Options& o, const uint32_t* sink, uint64_t words, uint64_t slice, uint64_t offset_words,
                          bool vector) {
  ReadCheck r;
  const bool l1 = o.workload == "l1";
  const uint64_t lanes = uint64_t(o.blocks) * o.threads;
  const uint64_t unit = vector ? 4 : 1;                      // words per access
  const uint64_t region = (l1 ? slice : words) / unit;       // accesses in the region
  const uint64_t region_lanes = l1 ? uint64_t(o.threads) : lanes;
  const uint64_t advance = (region_lanes * o.stride) % region;
  const uint64_t period = region / std::gcd(region, advance);
  const uint64_t steps = std::min(o.iterations, period);
  if (steps > 65536) return r;
  const unsigned sample_blocks = std::min(unsigned(o.blocks), 8U);
  for (unsigned sb = 0; sb < sample_blocks; ++sb) {
    const uint64_t block = sample_blocks == 1 ? 0 : uint64_t(sb) * (o.blocks - 1) / (sample_blocks - 1);
    for (int thread : {0, o.threads / 2, o.threads - 1}) {
      const uint64_t tid = l1 ? uint64_t(thread) : block * o.threads + thread;
      uint64_t pos = (tid * o.stride) % region;
      uint32_t cycle = 0, prefix = 0;
      for (uint64_t k = 0; k < steps; ++k) {
        uint32_t v = 0;
        for (uint64_t w = 0; w < unit; ++w)
        {
          const uint64_t index = offset_words + (l1 ? block * slice : 0) + pos * unit + w;
          v += o.fill == FILL_LCG ? lcg_word(index, o.seed) : random_word(index ^ o.seed);
        }
        cycle += v;
        if (k < o.iterations % period) prefix += v;
        pos = (pos + advance) % region;
      }
      const uint32_t expected = uint32_t(uint64_t(cycle) * (o.iterations / period)) + prefix;
      uint32_t actual = 0;
      check(cudaMemcpy(&actual, sink + block * o.threads + thread, 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
      ++r.checked;
      if (actual != expected) ++r.mismatched;
    }
  }
  r.status = r.mismatched ? "fail" : "pass";
  return r;
}

void experiment(Options o, const cudaDeviceProp& p, const Sink& out) {
  if (is_sfu(o.workload)) { experiment_sfu(o, p, out); return; }
  if (is_nonlinear(o.workload)) { experiment_nonlinear(o, p, out); return; }
  if (o.threads > p.maxThreadsPerBlock) throw Failure("thread count exceeds this device limit");
  if (!o.blocks) o.blocks = 2 * p.multiProcessorCount;
  if (o.blocks <= 0 || o.blocks > 1000000 || o.blocks > p.maxGridSize[0]) throw Failure("--blocks must be positive within practical/hardware limit");
  const bool latency = o.workload == "l2_latency";
  const bool lines = latency && o.chase_granularity == "line";
  const bool memory = o.workload == "l1" || o.workload == "l2" || o.workload == "hbm" || latency;
  const bool read = memory && !latency && o.access == "read";
  const bool vector = o.vector_bytes == 16;
  const bool tensor = o.workload == "tensor", gemm = o.workload == "gemm", control = o.workload == "control";
  if (tensor && o.threads != 128 && o.threads != 256) throw Failure("the tcgen05 tensor arm runs 128 or 256 threads per CTA");
  const uint64_t accesses_per_iteration = read || vector ? 1 : 4;
  const char* version = read ? (vector ? "vector_quad_single_stream_read_v1" : "scalar_single_stream_read_v3")
                      : memory && !latency ? (vector ? "vector_quad_copy_v1" : "scalar_four_stream_write_copy_v1")
                      : latency ? (lines ? "dependent_pointer_chain_lines_v1" : "dependent_pointer_chain_v1")
                      : tensor ? "tcgen05_tmem_operand_reuse_v1" : gemm ? "cublas_dense_gemm_v1" : "integer_issue_loop_v1";
  if (!o.iterations) o.iterations = gemm ? 1 : read ? 4096 : 1024;
  if (!o.batch_launches) o.batch_launches = gemm ? 1 : 16;
  if (!o.working_set_bytes) {
    if (o.workload == "l1") o.working_set_bytes = uint64_t(o.blocks) * 16 * 1024;
    else if (o.workload == "l2" || latency) o.working_set_bytes = std::max<uint64_t>(4, uint64_t(p.l2CacheSize) / 2 / 4 * 4);
    else o.working_set_bytes = std::max<uint64_t>(uint64_t(512) << 20, uint64_t(p.l2CacheSize) * 8);
  }
  const uint64_t requested_ws = o.working_set_bytes;
  const uint64_t lanes = uint64_t(o.blocks) * o.threads;
  const bool context = o.paired_reference && !control;
  const bool paired = context && !o.profile_region;
  // words: 32-bit payload words (line chase: 128-byte lines count as 32 words)
  uint64_t words = memory ? o.working_set_bytes / 4 : 1;
  if (lines) words = words / 32 * 32;
  if (memory && !latency && o.access != "read") {
    const uint64_t unit = vector ? 4 : 1;
    if (lanes > std::numeric_limits<uint64_t>::max() / (o.stride * unit)) throw Failure("write/copy ownership tile overflows");
    const uint64_t tile = lanes * o.stride * unit;
    words = words / tile * tile;
    if (!words) throw Failure("write/copy footprint must fit at least blocks*threads*stride 32-bit words");
  }
  if (read && vector) words = words / 4 * 4;
  uint64_t slice = o.workload == "l1" ? words / o.blocks : 0;
  if (memory && words == 0) throw Failure("memory footprint must contain at least one word");
  if (latency && !lines && words > std::numeric_limits<uint32_t>::max()) throw Failure("pointer chain exceeds uint32 node-index range");
  if (o.workload == "l1" && !slice) throw Failure("L1 footprint must contain at least one word per block");
  if (o.workload == "l1") words = slice * o.blocks;
  const uint64_t offset_words = memory ? o.offset_bytes / 4 : 0;
  if (memory && words + offset_words > uint64_t(p.totalGlobalMem) / 4 / (o.access == "read" ? 1 : 2) * 3 / 4)
    throw Failure("requested buffers exceed 75% of device capacity");
  const int acc = o.accumulators;
  const uint64_t tensor_out = tensor ? uint64_t(o.blocks) * kTmaM * tensor_tile_n(acc) : 1;
  const uint64_t a_count = gemm ? uint64_t(o.gemm_m) * o.gemm_k : tensor ? uint64_t(kTmaM) * kTmaK : 1;
  const uint64_t b_count = gemm ? uint64_t(o.gemm_k) * o.gemm_n : tensor ? uint64_t(256) * kTmaK : 1;
  const uint64_t c_count = gemm ? uint64_t(o.gemm_m) * o.gemm_n : tensor_out;
  DevBuf<uint32_t> input(memory ? words + offset_words : 1);
  DevBuf<uint32_t> output((memory && o.access != "read") ? words + offset_words : 1);
  DevBuf<uint32_t> sink(latency ? lanes : lanes);
  DevBuf<uint64_t> terminal(lines ? o.blocks : 1);
  DevBuf<uint16_t> a(a_count), b(b_count);
  DevBuf<float> c(c_count);
  DevBuf<unsigned char> mask(kSmSlots);
  DevBuf<unsigned long long> sm_blocks(kSmSlots), sm_cycles(kSmSlots), sm_loads(kSmSlots);
  DevBuf<uint32_t> ref_sink(context ? lanes : 1);
  DevBuf<unsigned long long> ref_blocks(context ? kSmSlots : 1);
  DevBuf<TensorStatus> tstatus(1);
  std::vector<unsigned char> mask_host(kSmSlots, o.sm_ids.empty() ? 1 : 0);
  for (unsigned id : o.sm_ids) mask_host[id] = 1;
  check(cudaMemcpy(mask.p, mask_host.data(), kSmSlots, cudaMemcpyHostToDevice), "cudaMemcpy");
  check(cudaMemset(sink.p, 0, lanes * 4), "cudaMemset");
  check(cudaMemset(c.p, 0, c_count * 4), "cudaMemset");
  for (auto* q : {sm_blocks.p, sm_cycles.p, sm_loads.p}) check(cudaMemset(q, 0, kSmSlots * 8), "cudaMemset");
  check(cudaMemset(ref_sink.p, 0, (context ? lanes : 1) * 4), "cudaMemset");
  check(cudaMemset(ref_blocks.p, 0, (context ? kSmSlots : 1) * 8), "cudaMemset");
  check(cudaMemset(tstatus.p, 0, sizeof(TensorStatus)), "cudaMemset");
  if (memory) check(launch_fill_words(input.p, words + offset_words, o.seed, p.multiProcessorCount, 0, o.fill), "fill");
  if (memory && o.access != "read")
    check(launch_fill_words(output.p, words + offset_words, o.seed ^ 0x9e3779b9ULL, p.multiProcessorCount, 0, o.fill), "fill");
  check(launch_fill_halves(a.p, a_count, o.seed, o.tensor_uniform, p.multiProcessorCount, 0), "fill");
  check(launch_fill_halves(b.p, b_count, o.seed ^ 12345ULL, o.tensor_uniform, p.multiProcessorCount, 0), "fill");
  check(cudaDeviceSynchronize(), "fill kernels");
  const bool filtered = !o.sm_ids.empty();
  const Admission adm{mask.p, filtered, sm_blocks.p}, ref_adm{mask.p, filtered, ref_blocks.p};
  uint64_t nodes = 0;
  if (latency) {
    // A full random cycle: std::mt19937_64(seed) + std::shuffle of 0..nodes-1 (gpu_bench.cu:722-731).
    nodes = lines ? words / 32 : words;
    std::vector<uint32_t> order(nodes);
    std::iota(order.begin(), order.end(), 0U);
    std::mt19937_64 gen(o.seed);
    std::shuffle(order.begin(), order.end(), gen);
    if (lines) {
      std::vector<uint64_t> host(nodes * 16, 0);
      for (uint64_t k = 0; k < nodes; ++k) host[uint64_t(order[k]) * 16] = order[(k + 1) % nodes];
      check(cudaMemcpy(input.p + offset_words, host.data(), nodes * 128, cudaMemcpyHostToDevice), "cudaMemcpy");
    } else {
      std::vector<uint32_t> host(nodes);
      for (uint64_t k = 0; k < nodes; ++k) host[order[k]] = order[(k + 1) % nodes];
      check(cudaMemcpy(input.p + offset_words, host.data(), nodes * 4, cudaMemcpyHostToDevice), "cudaMemcpy");
    }
  }
  if (o.workload == "l1") check(cudaFuncSetAttribute(kernel_symbol("read_scalar", 3, 1, 0), cudaFuncAttributePreferredSharedMemoryCarveout, 0), "carveout");
  // resources
  cudaFuncAttributes attr{};
  const void* handle = nullptr;
  const bool narrow = (o.workload == "l1" ? slice : words) <= 0xffffffffULL && o.iterations <= 0xffffffffULL;
  const int policy = o.read_cache_policy == "ca" ? RP_CA : o.read_cache_policy == "cs" ? RP_CS : RP_CG;
  if (o.workload == "l1") handle = kernel_symbol("read_scalar", 3, narrow, 0);
  else if (read) handle = vector ? kernel_symbol("read_vector", policy, 0, 0) : kernel_symbol("read_scalar", policy, narrow, 0);
  else if (memory && !latency) handle = vector ? kernel_symbol("copy_vector", 0, 0, 0) : kernel_symbol(o.access == "copy" ? "copy_scalar" : "write_scalar", 0, 0, 0);
  else if (latency) handle = kernel_symbol(lines ? "chase_lines" : "chase_words", 0, 0, 0);
  else if (control) handle = kernel_symbol("control", 0, 0, 0);
  bool have_resources = false;
  int max_blocks = 0;
  if (handle) {
    check(cudaFuncGetAttributes(&attr, handle), "cudaFuncGetAttributes");
    check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&max_blocks, handle, o.threads, 0), "occupancy");
    have_resources = true;
  } else if (tensor) {
    check(tensor_mma_attributes(acc, &attr), "cudaFuncGetAttributes");
    have_resources = true;
  }
  cublasHandle_t blas = nullptr;
  if (gemm) { check_blas(cublasCreate(&blas), "cublasCreate"); check_blas(cublasSetMathMode(blas, CUBLAS_TENSOR_OP_MATH), "cublasSetMathMode"); }
  uint64_t nonce = o.seed;
  const uint64_t quads = words / 4;
  auto single = [&] {
    ++nonce;
    const uint32_t* in = input.p + offset_words;
    if (tensor) check(launch_tensor_mma(a.p, b.p, c.p, o.iterations, acc, o.blocks, o.threads, adm, tstatus.p, 0), "tensor launch");
    else if (gemm) {
      const float alpha = 1.0f, beta = 0.0f;
      for (uint64_t k = 0; k < o.iterations; ++k)
        check_blas(cublasGemmEx(blas, CUBLAS_OP_N, CUBLAS_OP_N, o.gemm_m, o.gemm_n, o.gemm_k, &alpha, a.p, CUDA_R_16F, o.gemm_m,
                                b.p, CUDA_R_16F, o.gemm_k, &beta, c.p, CUDA_R_32F, o.gemm_m, CUBLAS_COMPUTE_32F,
                                CUBLAS_GEMM_DEFAULT_TENSOR_OP), "cublasGemmEx");
    } else if (control) check(launch_control(sink.p, o.iterations, o.blocks, o.threads, adm, 0), "control launch");
    else if (latency) {
      if (lines) check(launch_chase_lines(reinterpret_cast<const uint64_t*>(in), terminal.p, nodes, o.iterations, nonce,
                                          o.blocks, o.threads, adm, sm_cycles.p, sm_loads.p, 0), "chase launch");
      else check(launch_chase_words(in, sink.p, words, o.iterations, nonce, o.blocks, o.threads, adm, sm_cycles.p, sm_loads.p, 0), "chase launch");
    } else if (read) {
      if (vector) check(launch_read_vector(policy, in, sink.p, quads, o.stride, o.iterations, o.blocks, o.threads, adm, 0), "read launch");
      else check(launch_read_scalar(policy, o.workload == "l1", in, sink.p, words, slice, o.stride, o.iterations, o.blocks, o.threads, adm, 0), "read launch");
    } else {
      uint32_t* outp = output.p + offset_words;
      if (vector) check(launch_copy_vector(in, outp, sink.p, quads, o.stride, o.iterations, o.blocks, o.threads, adm, 0), "copy launch");
      else check(launch_write_copy_scalar(o.access == "copy", in, outp, sink.p, words, o.stride, o.iterations, o.blocks, o.threads, adm, 0), "write/copy launch");
    }
  };
  auto launch = [&] { for (int k = 0; k < o.batch_launches; ++k) single(); };
  auto ref_launch = [&] { for (int k = 0; k < o.batch_launches; ++k) check(launch_control(ref_sink.p, o.iterations, o.blocks, o.threads, ref_adm, 0), "control launch"); };
  out.line(protocol_json(o, paired, context, !gemm, "issue_loop",
                         "paired integer issue-loop operational contrast; launch geometry, iterations, SM admission mask and batching match; not isolated component energy"));
  run_phase(out, "warmup", o.warmup_seconds, o.warmup_batches, launch);
  idle_phase(out, "idle_pre", o.idle_seconds);
  std::vector<unsigned long long> seen(kSmSlots), ref_seen(kSmSlots);
  auto snapshot = [&]() -> uint64_t {
    if (gemm) return 0;
    check(cudaMemcpy(seen.data(), sm_blocks.p, kSmSlots * 8, cudaMemcpyDeviceToHost), "cudaMemcpy");
    return std::accumulate(seen.begin(), seen.end(), uint64_t(0));
  };
  auto ref_snapshot = [&]() -> uint64_t {
    check(cudaMemcpy(ref_seen.data(), ref_blocks.p, kSmSlots * 8, cudaMemcpyDeviceToHost), "cudaMemcpy");
    return std::accumulate(ref_seen.begin(), ref_seen.end(), uint64_t(0));
  };
  Timing t, rt;
  auto treatment_arm = [&] {
    if (paired) run_phase(out, "warmup_treatment", o.warmup_seconds, o.warmup_batches, launch);
    for (auto* q : {sm_blocks.p, sm_cycles.p, sm_loads.p}) check(cudaMemset(q, 0, kSmSlots * 8), "cudaMemset");
    nonce = o.seed;
    t = run_phase(out, "measure", o.seconds, o.fixed_batches, launch, snapshot, o.profile_region);
  };
  auto reference_arm = [&] {
    run_phase(out, "warmup_reference", o.warmup_seconds, o.warmup_batches, ref_launch);
    check(cudaMemset(ref_blocks.p, 0, kSmSlots * 8), "cudaMemset");
    rt = run_phase(out, "active_reference", o.seconds, o.fixed_batches, ref_launch, ref_snapshot);
  };
  if (paired && o.reference_order == "AB") reference_arm();
  treatment_arm();
  if (paired && o.reference_order == "BA") reference_arm();
  idle_phase(out, "idle_post", o.idle_seconds);
  if (paired) {
    check(cudaMemcpy(ref_seen.data(), ref_blocks.p, kSmSlots * 8, cudaMemcpyDeviceToHost), "cudaMemcpy");
    const uint64_t admitted = std::accumulate(ref_seen.begin(), ref_seen.end(), uint64_t(0));
    if (!admitted) throw Failure("no active-reference blocks were admitted by the SM filter");
    std::vector<unsigned> missing;
    for (unsigned id : o.sm_ids) if (!ref_seen[id]) missing.push_back(id);
    Obj j;
    j.str("type", "active_reference_result").str("workload", "control").str("reference_kind", "issue_loop")
     .str("kernel_implementation_version", "integer_issue_loop_v1").str("block_completion_count_source", "per_sm_admission_atomics")
     .str("active_sm_distribution_status", "admission_counter_observed")
     .f("duration_s", rt.device_s).f("host_duration_s", rt.host_s).u("batches", rt.batches).i("batch_launches", o.batch_launches)
     .u("iterations_per_launch", o.iterations).i("blocks", o.blocks).i("threads", o.threads).u("admitted_blocks", admitted)
     .u("operations", 0).u("logical_bytes", 0).str("operation_unit", "not FLOPs or target bytes; integer issue-loop reference")
     .raw("measure_epochs", epochs_json(rt, o.batch_launches, [](Obj& e, const Epoch&) { e.u("operations", 0).u("logical_bytes", 0); }))
     .raw("sanity", Obj().b("requested_sm_coverage_complete", missing.empty()).done());
    out.line(j.done());
    if (!missing.empty()) throw Failure("requested active-reference SM coverage incomplete; reject this trial");
  }
  // admissions, counts
  std::vector<unsigned long long> observed(kSmSlots);
  check(cudaMemcpy(observed.data(), sm_blocks.p, kSmSlots * 8, cudaMemcpyDeviceToHost), "cudaMemcpy");
  uint64_t admitted = 0;
  std::vector<unsigned> active, missing;
  for (unsigned id = 0; id < kSmSlots; ++id) if (observed[id]) { active.push_back(id); admitted += observed[id]; }
  if (!gemm && !admitted) throw Failure("no blocks were admitted by the SM filter");
  for (unsigned id : o.sm_ids) if (!observed[id]) missing.push_back(id);
  TensorStatus ts{};
  if (tensor) check(cudaMemcpy(&ts, tstatus.p, sizeof ts, cudaMemcpyDeviceToHost), "cudaMemcpy");
  auto counts = [&](uint64_t adm_blocks, uint64_t batches, long double* ops, long double* bytes) {
    *ops = 0; *bytes = 0;
    if (tensor) *ops = (long double)adm_blocks * o.iterations * tensor_flops_per_iteration(acc);
    else if (gemm) *ops = (long double)batches * o.batch_launches * o.iterations * 2.0L * o.gemm_m * o.gemm_n * o.gemm_k;
    else if (latency) { *ops = (long double)adm_blocks * o.iterations; *bytes = *ops * (lines ? 8 : 4); }
    else if (memory) {
      *ops = (long double)adm_blocks * o.threads * o.iterations * accesses_per_iteration;
      *bytes = *ops * (vector ? 16 : 4) * (o.access == "copy" ? 2 : 1);
    }
  };
  long double operations, logical_bytes;
  counts(admitted, t.batches, &operations, &logical_bytes);
  // checks
  uint64_t checksum = 0;
  bool finite = true;
  ReadCheck rc;
  const char* checksum_kind = "uint32_sink_sample";
  if (read && !filtered) {
    rc = check_read_sums(o, sink.p, words, slice, offset_words, vector);
    finite = rc.mismatched == 0;
  } else if (read) rc.status = "not_checked_sm_filtered";
  if (tensor || gemm) {
    std::vector<float> sample(std::min<uint64_t>(256, c_count));
    check(cudaMemcpy(sample.data(), c.p, sample.size() * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
    for (float v : sample) { uint32_t bits; memcpy(&bits, &v, 4); checksum = checksum * 1315423911ULL + bits; finite = finite && std::isfinite(v); }
    checksum_kind = "fp32_output_sample_hash";
    if (tensor && ts.timeouts) finite = false;
  } else if (lines) {
    std::vector<uint64_t> term(o.blocks);
    check(cudaMemcpy(term.data(), terminal.p, o.blocks * 8, cudaMemcpyDeviceToHost), "cudaMemcpy");
    for (uint64_t w : term) checksum = checksum * 1315423911ULL + w;
    checksum_kind = "chain_terminal_node_hash";
  } else {
    std::vector<uint32_t> sample(std::min<uint64_t>(1024, lanes));
    check(cudaMemcpy(sample.data(), sink.p, sample.size() * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
    checksum = checksum_words(sample);
    if (read) checksum_kind = vector ? "sum32_vector_reads_per_thread_sample_hash" : "sum32_scalar_reads_per_thread_sample_hash";
  }
  std::vector<unsigned long long> cycles(kSmSlots), loads(kSmSlots);
  if (latency) {
    check(cudaMemcpy(cycles.data(), sm_cycles.p, kSmSlots * 8, cudaMemcpyDeviceToHost), "cudaMemcpy");
    check(cudaMemcpy(loads.data(), sm_loads.p, kSmSlots * 8, cudaMemcpyDeviceToHost), "cudaMemcpy");
  }
  Obj j;
  j.str("type", "result").str("workload", o.workload).str("access", o.access)
   .f("duration_s", t.device_s).f("host_duration_s", t.host_s).u("batches", t.batches).u("iterations_per_launch", o.iterations)
   .u("iterations_per_batch", o.iterations * o.batch_launches).i("batch_launches", o.batch_launches)
   .u("workload_launches", t.batches * o.batch_launches)
   .raw("kernel_launches", gemm ? "null" : std::to_string(t.batches * o.batch_launches))
   .u("gemm_invocations", gemm ? t.batches * o.batch_launches * o.iterations : 0)
   .u("fixed_batches", o.fixed_batches).u("warmup_batches", o.warmup_batches)
   .f("mean_batch_duration_s", t.device_s / double(std::max<uint64_t>(1, t.batches)))
   .str("duration_scope", "CUDA event elapsed experiment window including gaps; not summed kernel busy time")
   .str("kernel_implementation_version", version)
   .raw("grid_mode", "null").raw("input_elements", "null")
   .str("block_completion_count_source", gemm ? "not_applicable" : "per_sm_admission_atomics")
   .raw("memory_accesses_per_thread_iteration", memory && !latency ? std::to_string(accesses_per_iteration) : "null")
   .raw("memory_read_checksum_scope", read ? "\"sum32_of_all_reads_per_thread\"" : "null")
   .raw("read_cache_policy", read ? quoted(o.read_cache_policy) : "null")
   .raw("memory_read_index_math", read ? quoted(narrow && !vector ? "uint32" : "uint64") : "null")
   .raw("memory_read_validation", read ? Obj().str("status", rc.status).u("checked_values", rc.checked).u("mismatched_values", rc.mismatched)
        .str("scope", "CPU deterministic input/index oracle for modulo-2^32 sums at up to eight CTAs and three threads per CTA; repeated address cycles folded").done() : "null")
   .f("operations", double(operations))
   .str("operation_unit", memory ? (vector ? "16-byte memory accesses (copy pairs count once)" : "32-bit memory accesses (copy pairs count once)") : control ? "not attributed" : "dense FP FLOPs (FMA=2)")
   .f("logical_bytes", double(logical_bytes)).f("throughput_ops_s", double(operations) / t.device_s)
   .f("throughput_bytes_s", double(logical_bytes) / t.device_s).i("blocks", o.blocks).i("threads", o.threads)
   .b("launch_geometry_applies", !gemm).u("admitted_blocks", admitted)
   .u("working_set_bytes", memory ? words * 4 : 0).u("requested_working_set_bytes", memory ? requested_ws : 0)
   .raw("write_copy_thread_addresses_disjoint", memory && !latency && o.access != "read" ? "true" : "null")
   .u("l1_bytes_per_block", slice * 4).u("stride_elements", o.stride).u("offset_bytes", o.offset_bytes)
   .raw("memory_word_bytes", memory ? "4" : "null").raw("stride_words", memory ? std::to_string(o.stride) : "null")
   .raw("lane_stride_bytes", memory ? std::to_string(o.stride * (vector ? 16 : 4)) : "null")
   .i("memory_vector_bytes", memory ? o.vector_bytes : 0).str("chase_granularity", o.chase_granularity)
   .raw("memory_fill", memory ? (o.fill == FILL_LCG ? "\"uint32_lcg_1664525_1013904223_v1\"" : "\"random_word_xor_seed_v1\"") : "null")
   .i("tensor_accumulators", acc).i("tensor_tile_m", tensor ? kTmaM : 0).i("tensor_tile_n", tensor ? tensor_tile_n(acc) : 0)
   .i("gemm_m", o.gemm_m).i("gemm_n", o.gemm_n).i("gemm_k", o.gemm_k).u("seed", o.seed)
   .u("checksum", checksum).str("checksum_kind", checksum_kind)
   .raw("kernel_resources", have_resources ? resources_json(attr, max_blocks, o.threads, p, o.blocks) : "null")
   .raw("numerical_validation", Obj().u("checked_values", 0).f("max_absolute_error", 0).f("max_relative_error", 0).done())
   .raw("sanity", Obj().b("finite_output_sample", finite)
                       .raw("memory_read_sample_matches_reference", read && rc.checked ? (rc.mismatched ? "false" : "true") : "null")
                       .raw("numerical_validation_passed", "null").b("requested_sm_coverage_complete", missing.empty()).done())
   .b("profile_region", o.profile_region).b("paired_reference_context_allocated", context);
  if (tensor) j.raw("tensor_status", Obj().u("bounded_wait_timeouts", ts.timeouts).u("completed_ctas", ts.done_ctas).done());
  j.raw("measure_epochs", epochs_json(t, o.batch_launches, [&](Obj& e, const Epoch& ep) {
    long double eo, eb;
    counts(ep.admitted, ep.batches, &eo, &eb);
    e.f("operations", double(eo)).f("logical_bytes", double(eb));
  }));
  std::string ids = "[";
  for (size_t k = 0; k < active.size(); ++k) ids += (k ? "," : "") + std::to_string(active[k]);
  j.raw("active_sm_ids", ids + "]").str("active_sm_distribution_status", gemm ? "not_measured_gemm" : "admission_counter_observed");
  std::string miss = "[";
  for (size_t k = 0; k < missing.size(); ++k) miss += (k ? "," : "") + std::to_string(missing[k]);
  j.raw("missing_requested_sm_ids", miss + "]");
  Obj probe;
  probe.b("enabled", latency).str("scope", lines ? "dependent 64-bit links on 128-byte lines, one chain per block" : "dependent .cg chain, one lane per admitted block");
  std::string per_sm = "{";
  if (latency) {
    bool first = true;
    for (unsigned id : active) {
      per_sm += (first ? "" : ",") + quoted(std::to_string(id)) + ":" +
                Obj().u("loads", loads[id]).u("cycles", cycles[id]).f("cycles_per_access", loads[id] ? double(cycles[id]) / loads[id] : 0).done();
      first = false;
    }
  }
  probe.raw("per_sm", per_sm + "}");
  j.raw("latency_probe", probe.done()).str("sparsity", "dense")
   .str("input_precision", "fp16 for tensor/gemm; uint32 memory payload otherwise").str("accumulator_precision", "fp32");
  out.line(j.done());
  if (blas) cublasDestroy(blas);
  if (tensor && ts.timeouts) throw Failure("tensor arm: a bounded device wait timed out");
  if (!finite) throw Failure("non-finite or numerically incorrect output sample");
  if (!missing.empty()) throw Failure("requested SM coverage incomplete; reject this trial");
}

}  // namespace
}  // namespace pm

using namespace pm;

extern "C" int pm_tensor_probe(int accumulators, uint64_t iterations, int uniform, uint64_t seed, float* out,
                               size_t out_count, uint16_t* a_out, uint16_t* b_out) {
  if (accumulators < 1 || accumulators > 8 || !out) return fail(PM_E_INVALID, "pm_tensor_probe: bad arguments");
  const int n = tensor_tile_n(accumulators);
  if (out_count < size_t(kTmaM) * n) return fail(PM_E_INVALID, "pm_tensor_probe: out needs 128*N floats");
  try {
    int sms = 0;
    check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0), "attr");
    DevBuf<uint16_t> a(size_t(kTmaM) * kTmaK), b(size_t(256) * kTmaK);
    DevBuf<float> c(size_t(kTmaM) * n);
    DevBuf<unsigned char> mask(kSmSlots);
    DevBuf<unsigned long long> blocks(kSmSlots);
    DevBuf<TensorStatus> st(1);
    check(cudaMemset(mask.p, 1, kSmSlots), "cudaMemset");
    check(cudaMemset(blocks.p, 0, kSmSlots * 8), "cudaMemset");
    check(cudaMemset(st.p, 0, sizeof(TensorStatus)), "cudaMemset");
    check(cudaMemset(c.p, 0, size_t(kTmaM) * n * 4), "cudaMemset");
    check(launch_fill_halves(a.p, size_t(kTmaM) * kTmaK, seed, uniform, sms, 0), "fill");
    check(launch_fill_halves(b.p, size_t(256) * kTmaK, seed ^ 12345ULL, uniform, sms, 0), "fill");
    check(launch_tensor_mma(a.p, b.p, c.p, iterations, accumulators, 1, 128, Admission{mask.p, false, blocks.p}, st.p, 0), "tensor launch");
    check(cudaDeviceSynchronize(), "tensor kernel");
    TensorStatus ts{};
    check(cudaMemcpy(&ts, st.p, sizeof ts, cudaMemcpyDeviceToHost), "cudaMemcpy");
    if (ts.timeouts) return fail(PM_E_TIMEOUT, "tensor probe: bounded wait gave up");
    check(cudaMemcpy(out, c.p, size_t(kTmaM) * n * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
    if (a_out) check(cudaMemcpy(a_out, a.p, size_t(kTmaM) * kTmaK * 2, cudaMemcpyDeviceToHost), "cudaMemcpy");
    if (b_out) check(cudaMemcpy(b_out, b.p, size_t(256) * kTmaK * 2, cudaMemcpyDeviceToHost), "cudaMemcpy");
    return PM_OK;
  } catch (const std::exception& e) {
    return fail(PM_E_CUDA, "%s", e.what());
  }
}

extern "C" int pm_gemm_probe(int m, int n, int k, int uniform, uint64_t seed, float* out, uint16_t* a_out,
                             uint16_t* b_out) {
  if (m <= 0 || n <= 0 || k <= 0 || m > 4096 || n > 4096 || k > 4096 || !out)
    return fail(PM_E_INVALID, "pm_gemm_probe: dimensions must be 1..4096 and out non-NULL");
  try {
    int sms = 0;
    check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0), "attr");
    DevBuf<uint16_t> a(size_t(m) * k), b(size_t(k) * n);
    DevBuf<float> c(size_t(m) * n);
    // The gemm arm's operands and call: column-major A (m x k) and B (k x n)
    // filled as the arm fills them, fp32 C from cublasGemmEx on the tensor cores.
    check(launch_fill_halves(a.p, size_t(m) * k, seed, uniform, sms, 0), "fill");
    check(launch_fill_halves(b.p, size_t(k) * n, seed ^ 12345ULL, uniform, sms, 0), "fill");
    cublasHandle_t blas = nullptr;
    check_blas(cublasCreate(&blas), "cublasCreate");
    const float alpha = 1.0f, beta = 0.0f;
    cublasStatus_t st = cublasSetMathMode(blas, CUBLAS_TENSOR_OP_MATH);
    if (st == CUBLAS_STATUS_SUCCESS)
      st = cublasGemmEx(blas, CUBLAS_OP_N, CUBLAS_OP_N, m, n, k, &alpha, a.p, CUDA_R_16F, m, b.p, CUDA_R_16F, k, &beta,
                        c.p, CUDA_R_32F, m, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT_TENSOR_OP);
    cublasDestroy(blas);
    check_blas(st, "cublasGemmEx");
    check(cudaDeviceSynchronize(), "gemm");
    check(cudaMemcpy(out, c.p, size_t(m) * n * 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
    if (a_out) check(cudaMemcpy(a_out, a.p, size_t(m) * k * 2, cudaMemcpyDeviceToHost), "cudaMemcpy");
    if (b_out) check(cudaMemcpy(b_out, b.p, size_t(k) * n * 2, cudaMemcpyDeviceToHost), "cudaMemcpy");
    return PM_OK;
  } catch (const std::exception& e) {
    return fail(PM_E_CUDA, "%s", e.what());
  }
}

extern "C" int pm_powerbench(int argc, const char* const* argv, pm_line_cb cb, void* user) {
  if (!cb || argc < 1 || !argv) return fail(PM_E_INVALID, "pm_powerbench: NULL argument");
  const Sink out{cb, user};
  try {
    bool help = false;
    Options o = parse_options(argc, argv, out, &help);
    if (help) { out.line(std::string("#") + kUsage); return 0; }
    check(cudaSetDevice(o.device), "cudaSetDevice");
    cudaDeviceProp p{};
    check(cudaGetDeviceProperties(&p, o.device), "cudaGetDeviceProperties");
    describe(o, p, out);
    if (!o.describe) experiment(o, p, out);
    return 0;
  } catch (const std::exception& e) {
    fail(1, "%s", e.what());
    return 1;
  }
}
