// accessor_dot_bench -- FP32-storage DOT over the dot_v1 datasets through
// libautdot, with the flags, modes and CSV schemas of the reference's
// src/accessor_dot_bench.cu (options :127-300, performance CSV :544-612,
// accuracy CSV :714-770, profile CSV :772-824).
//
// Variants keep the reference's names; each maps to the fused DOT of FP32
// storage:
//   raw_f32 / accessor_f32_f32   AUT_ACCUM_FP32 (raw: LDG strategy,
//   raw_f64 / accessor_f64_f32   AUT_ACCUM_FP64  accessor: TMA strategy)
// The result is always an FP64 (the library's FP32 accumulation of raw FP32
// storage is compensated, see autdot.h), so `result_bits` holds the 16 hex
// digits of that double for every variant.  Inputs come from the device
// generator of the dot_v1 cases (aut_generate_dot_v1, bit-identical to the
// reference's); the accuracy reference is the same compensated long-double
// sum over the host generator (include/aut/dot_dataset.hpp).
#include <autdot.h>

#include "aut/dot_dataset.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <limits>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void aut_check(aut_status s, const char *what) {
  if (s != AUT_OK) throw std::runtime_error(std::string(what) + ": " + aut_last_error());
}

enum class mode { performance, accuracy, profile };
enum class variant { raw_f32, raw_f64, accessor_f32_f32, accessor_f64_f32 };
constexpr std::array<variant, 4> all_variants{variant::raw_f32, variant::raw_f64,
                                              variant::accessor_f32_f32,
                                              variant::accessor_f64_f32};

const char *name_of(mode m) {
  return m == mode::performance ? "performance" : m == mode::accuracy ? "accuracy" : "profile";
}
const char *name_of(variant v) {
  switch (v) {
  case variant::raw_f32: return "raw_f32";
  case variant::raw_f64: return "raw_f64";
  case variant::accessor_f32_f32: return "accessor_f32_f32";
  case variant::accessor_f64_f32: return "accessor_f64_f32";
  }
  return "unknown";
}
bool fp64(variant v) { return v == variant::raw_f64 || v == variant::accessor_f64_f32; }
bool raw(variant v) { return v == variant::raw_f32 || v == variant::raw_f64; }

struct options {
  mode run_mode{mode::performance};
  bool every_variant{true};
  variant one{variant::raw_f32};
  std::vector<int> powers;
  std::size_t exact_count{0};
  int warmup{5}, rounds{3}, samples{20}, iterations{0};
  double target_sample_ms{50.0};
  std::string dataset{aut::dataset::performance_case.id};
  std::string output{"-"};
};

std::vector<int> int_list(const std::string &text) {
  std::vector<int> out;
  std::stringstream ss(text);
  std::string t;
  while (std::getline(ss, t, ',')) {
    if (t.empty()) throw std::runtime_error("empty item in integer list: " + text);
    out.push_back(std::stoi(t));
  }
  if (out.empty()) throw std::runtime_error("integer list must not be empty");
  return out;
}

void usage(const char *program) {
  std::cout << "Usage: " << program << " [options]\n"
            << "  --mode performance|accuracy|profile\n"
            << "  --variant all|raw_f32|raw_f64|accessor_f32_f32|accessor_f64_f32\n"
            << "  --powers P[,P...]   sizes 2^P (default: accuracy 10,16,20; "
               "performance 10,16,20,23,26,27)\n"
            << "  --n N               one exact size (instead of --powers)\n"
            << "  --warmup W --rounds R --samples S --iterations I "
               "--target-sample-ms T\n"
            << "  --dataset ID        dot_v1 case for performance/profile\n"
            << "  --output PATH|-\n";
}

options parse(int argc, char **argv, bool &help) {
  options o;
  bool powers_set = false;
  help = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto value = [&]() -> std::string {
      if (++i >= argc) throw std::runtime_error("missing value after " + a);
      return argv[i];
    };
    if (a == "--help" || a == "-h") {
      help = true;
    } else if (a == "--mode") {
      const auto v = value();
      if (v == "performance") o.run_mode = mode::performance;
      else if (v == "accuracy") o.run_mode = mode::accuracy;
      else if (v == "profile") o.run_mode = mode::profile;
      else throw std::runtime_error("unknown mode: " + v);
    } else if (a == "--variant") {
      const auto v = value();
      if (v == "all") {
        o.every_variant = true;
      } else {
        o.every_variant = false;
        bool found = false;
        for (auto c : all_variants)
          if (v == name_of(c)) o.one = c, found = true;
        if (!found) throw std::runtime_error("unknown variant: " + v);
      }
    } else if (a == "--powers") {
      o.powers = int_list(value());
      powers_set = true;
    } else if (a == "--n") {
      std::size_t used = 0;
      const std::string v = value();
      o.exact_count = std::stoull(v, &used, 0);
      if (used != v.size() || o.exact_count == 0)
        throw std::runtime_error("expected a positive integer: " + v);
    } else if (a == "--warmup") o.warmup = std::stoi(value());
    else if (a == "--rounds") o.rounds = std::stoi(value());
    else if (a == "--samples") o.samples = std::stoi(value());
    else if (a == "--iterations") o.iterations = std::stoi(value());
    else if (a == "--target-sample-ms") o.target_sample_ms = std::stod(value());
    else if (a == "--dataset") o.dataset = value();
    else if (a == "--output") o.output = value();
    else throw std::runtime_error("unknown argument: " + a);
  }
  if (o.warmup < 0 || o.rounds <= 0 || o.samples <= 0 || o.iterations < 0 ||
      o.target_sample_ms <= 0.0)
    throw std::runtime_error("warmup must be nonnegative; rounds, samples, and target time "
                             "must be positive; iterations must be nonnegative");
  if (o.exact_count != 0 && powers_set)
    throw std::runtime_error("--n and --powers are mutually exclusive");
  if (o.run_mode == mode::profile && o.every_variant)
    throw std::runtime_error("profile mode requires one explicit --variant");
  if (!powers_set)
    o.powers = o.run_mode == mode::accuracy ? std::vector<int>{10, 16, 20}
                                            : std::vector<int>{10, 16, 20, 23, 26, 27};
  for (int p : o.powers)
    if (p < 0 || p > 30) throw std::runtime_error("powers must be in [0, 30]");
  return o;
}

std::vector<std::size_t> sizes(const options &o) {
  if (o.exact_count != 0) return {o.exact_count};
  std::vector<std::size_t> out;
  for (int p : o.powers) out.push_back(std::size_t{1} << p);
  return out;
}

const aut::dataset::case_spec &find_case(const std::string &id) {
  for (const auto &c : aut::dataset::accuracy_cases)
    if (id == c.id) return c;
  throw std::runtime_error("unknown dataset: " + id);
}

struct environment {
  std::string gpu;
  int major = 0, minor = 0, sms = 0, runtime = 0, driver = 0;
};

environment probe(int device) {
  environment e;
  cudaDeviceProp p{};
  cuda_check(cudaGetDeviceProperties(&p, device), "cudaGetDeviceProperties");
  e.gpu = p.name;
  e.major = p.major;
  e.minor = p.minor;
  e.sms = p.multiProcessorCount;
  cuda_check(cudaRuntimeGetVersion(&e.runtime), "cudaRuntimeGetVersion");
  cuda_check(cudaDriverGetVersion(&e.driver), "cudaDriverGetVersion");
  return e;
}

void write_env(std::ostream &out, const environment &e) {
  out << e.gpu << ',' << e.major << '.' << e.minor << ',' << e.sms << ',' << e.runtime << ','
      << e.driver;
}

// one device buffer pair holding a dot_v1 case of `count` values
struct inputs {
  float *x = nullptr, *y = nullptr;
  double *result = nullptr;
  std::size_t count = 0;
  inputs(const aut::dataset::parameters &spec, std::size_t n, cudaStream_t s) : count(n) {
    cuda_check(cudaMalloc(&x, std::max<std::size_t>(n, 4) * sizeof(float)), "cudaMalloc");
    cuda_check(cudaMalloc(&y, std::max<std::size_t>(n, 4) * sizeof(float)), "cudaMalloc");
    cuda_check(cudaMalloc(&result, sizeof(double)), "cudaMalloc");
    const int family = static_cast<int>(spec.kind);
    aut_check(aut_generate_dot_v1(family, spec.seed, spec.parameter, 0, n, 0, n, x, s),
              "aut_generate_dot_v1");
    aut_check(aut_generate_dot_v1(family, spec.seed, spec.parameter, 1, n, 0, n, y, s),
              "aut_generate_dot_v1");
    cuda_check(cudaStreamSynchronize(s), "generate");
  }
  ~inputs() {
    cudaFree(x);
    cudaFree(y);
    cudaFree(result);
  }
};

void launch(aut_workspace *ws, variant v, const inputs &in, cudaStream_t s) {
  aut_check(aut_dot_strategy(ws, aut_format_id("fp32"), AUT_LAYOUT_DENSE,
                             fp64(v) ? AUT_ACCUM_FP64 : AUT_ACCUM_FP32,
                             raw(v) ? AUT_STRATEGY_LDG : AUT_STRATEGY_TMA, in.x, in.y, in.count,
                             in.result, s),
            "aut_dot_strategy");
}

float elapsed_ms(aut_workspace *ws, variant v, const inputs &in, cudaStream_t s, int iterations) {
  cudaEvent_t a, b;
  cuda_check(cudaEventCreate(&a), "cudaEventCreate");
  cuda_check(cudaEventCreate(&b), "cudaEventCreate");
  cuda_check(cudaEventRecord(a, s), "cudaEventRecord");
  for (int i = 0; i < iterations; ++i) launch(ws, v, in, s);
  cuda_check(cudaEventRecord(b, s), "cudaEventRecord");
  cuda_check(cudaEventSynchronize(b), "cudaEventSynchronize");
  float ms = 0.f;
  cuda_check(cudaEventElapsedTime(&ms, a, b), "cudaEventElapsedTime");
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return ms;
}

int calibrate(const options &o, aut_workspace *ws, variant v, const inputs &in, cudaStream_t s) {
  if (o.iterations > 0) return o.iterations;
  const float one = std::max(elapsed_ms(ws, v, in, s, 1), 1e-4f);
  return std::clamp(static_cast<int>(std::ceil(o.target_sample_ms / one)), 1, 1 << 20);
}

double result_of(const inputs &in, cudaStream_t s) {
  double r = 0.0;
  cuda_check(cudaMemcpyAsync(&r, in.result, sizeof r, cudaMemcpyDeviceToHost, s), "copy");
  cuda_check(cudaStreamSynchronize(s), "sync");
  return r;
}

std::string bits_of(double v) {
  std::uint64_t b;
  std::memcpy(&b, &v, sizeof b);
  std::ostringstream o;
  o << "0x" << std::hex << std::setfill('0') << std::setw(16) << b;
  return o.str();
}

std::vector<variant> chosen(const options &o) {
  if (o.every_variant) return {all_variants.begin(), all_variants.end()};
  return {o.one};
}

void performance(const options &o, const environment &env, aut_workspace *ws, cudaStream_t s,
                 std::ostream &out) {
  out << "gpu,compute_capability,multiprocessors,cuda_runtime,cuda_driver,"
         "dataset,variant,storage_type,arithmetic_type,access_kind,n,"
         "algorithmic_bytes,algorithmic_flops,"
         "arithmetic_intensity_flop_per_byte,blocks,threads,round,"
         "order_in_round,iterations,sample,total_time_ms,giga_elements_per_s,"
         "algorithmic_gb_per_s,gflop_per_s\n";
  const auto &spec = find_case(o.dataset);
  const auto vs = chosen(o);
  int32_t sm_count = 0, max_blocks = 0;
  aut_check(aut_workspace_info(ws, &sm_count, &max_blocks), "aut_workspace_info");
  const auto list = sizes(o);
  for (std::size_t ci = 0; ci < list.size(); ++ci) {
    const inputs in(spec.values, list[ci], s);
    std::vector<int> iters(vs.size());
    for (std::size_t k = 0; k < vs.size(); ++k) {
      for (int w = 0; w < o.warmup; ++w) launch(ws, vs[k], in, s);
      cuda_check(cudaStreamSynchronize(s), "warmup");
      iters[k] = calibrate(o, ws, vs[k], in, s);
    }
    for (int round = 0; round < o.rounds; ++round) {
      const std::size_t rotation = (ci + static_cast<std::size_t>(round)) % vs.size();
      for (std::size_t order = 0; order < vs.size(); ++order) {
        const std::size_t k = (order + rotation) % vs.size();
        for (int sample = 0; sample < o.samples; ++sample) {
          const double op_ms = static_cast<double>(elapsed_ms(ws, vs[k], in, s, iters[k])) /
                               iters[k];
          const double sec = op_ms * 1e-3;
          const double bytes = 8.0 * static_cast<double>(in.count);
          const double flops = 2.0 * static_cast<double>(in.count);
          write_env(out, env);
          out << ',' << spec.id << ',' << name_of(vs[k]) << ",float32,"
              << (fp64(vs[k]) ? "float64" : "float32") << ',' << (raw(vs[k]) ? "raw" : "accessor")
              << ',' << in.count << ',' << std::setprecision(17) << bytes << ',' << flops
              << ",0.25," << sm_count << ",256," << round << ',' << order << ',' << iters[k]
              << ',' << sample << ',' << op_ms << ','
              << static_cast<double>(in.count) / sec / 1e9 << ',' << bytes / sec / 1e9 << ','
              << flops / sec / 1e9 << '\n';
        }
        out.flush();
      }
    }
    std::cerr << "Performance N=" << in.count << " complete\n";
  }
}

// The reference's compensated long-double sum (src/accessor_dot_bench.cu:
// 615-638): a running sum plus the rounding error of every addition.
struct compensated {
  long double sum = 0.0L, correction = 0.0L;
  void add(long double v) {
    const long double next = sum + v;
    correction += std::fabs(sum) >= std::fabs(v) ? (sum - next) + v : (v - next) + sum;
    sum = next;
  }
  long double value() const { return sum + correction; }
};

void accuracy(const options &o, const environment &env, aut_workspace *ws, cudaStream_t s,
              std::ostream &out) {
  out << "gpu,compute_capability,multiprocessors,cuda_runtime,cuda_driver,"
         "dataset,variant,storage_type,arithmetic_type,access_kind,n,blocks,"
         "threads,result,result_bits,reference,absolute_error,relative_error,"
         "normalized_error,dot_condition_number,x_fingerprint,"
         "y_fingerprint,finite\n";
  int32_t sm_count = 0, max_blocks = 0;
  aut_check(aut_workspace_info(ws, &sm_count, &max_blocks), "aut_workspace_info");
  for (const auto &c : aut::dataset::accuracy_cases) {
    for (const auto count : sizes(o)) {
      const inputs in(c.values, count, s);
      compensated dot, sabs;
      std::uint64_t fx = 1469598103934665603ULL, fy = 1469598103934665603ULL;
      for (std::size_t i = 0; i < count; ++i) {
        const float x = aut::dataset::value(c.values, 0, i, count);
        const float y = aut::dataset::value(c.values, 1, i, count);
        std::uint32_t bx, by;
        std::memcpy(&bx, &x, 4);
        std::memcpy(&by, &y, 4);
        fx = (fx ^ bx) * 1099511628211ULL;
        fy = (fy ^ by) * 1099511628211ULL;
        const long double p = static_cast<long double>(x) * static_cast<long double>(y);
        dot.add(p);
        sabs.add(std::fabs(p));
      }
      const long double ref = dot.value(), ref_abs = sabs.value();
      for (const auto v : chosen(o)) {
        for (int w = 0; w < o.warmup; ++w) launch(ws, v, in, s);
        cuda_check(cudaStreamSynchronize(s), "warmup");
        launch(ws, v, in, s);
        const double got = result_of(in, s);
        const long double abs_err = std::fabs(static_cast<long double>(got) - ref);
        const long double nan = std::numeric_limits<long double>::quiet_NaN();
        write_env(out, env);
        out << ',' << c.id << ',' << name_of(v) << ",float32,"
            << (fp64(v) ? "float64" : "float32") << ',' << (raw(v) ? "raw" : "accessor") << ','
            << count << ',' << sm_count << ",256," << std::setprecision(21)
            << static_cast<long double>(got) << ',' << bits_of(got) << ',' << ref << ','
            << abs_err << ',' << (ref == 0.0L ? nan : abs_err / std::fabs(ref)) << ','
            << (ref_abs == 0.0L ? nan : abs_err / ref_abs) << ','
            << (ref == 0.0L ? std::numeric_limits<long double>::infinity()
                            : ref_abs / std::fabs(ref))
            << ",0x" << std::hex << fx << ",0x" << fy << std::dec << ','
            << (std::isfinite(got) ? "true" : "false") << '\n';
      }
      out.flush();
      std::cerr << "Accuracy " << c.id << " N=" << count << " complete\n";
    }
  }
}

void profile(const options &o, const environment &env, aut_workspace *ws, cudaStream_t s,
             std::ostream &out) {
  const auto list = sizes(o);
  if (list.size() != 1) throw std::runtime_error("profile mode requires exactly one size");
  const auto &spec = find_case(o.dataset);
  const inputs in(spec.values, list.front(), s);
  for (int w = 0; w < o.warmup; ++w) launch(ws, o.one, in, s);
  cuda_check(cudaStreamSynchronize(s), "warmup");
  launch(ws, o.one, in, s);
  const double got = result_of(in, s);
  int32_t sm_count = 0, max_blocks = 0;
  aut_check(aut_workspace_info(ws, &sm_count, &max_blocks), "aut_workspace_info");
  out << "gpu,compute_capability,multiprocessors,cuda_runtime,cuda_driver,"
         "mode,dataset,variant,storage_type,arithmetic_type,access_kind,n,"
         "algorithmic_bytes,algorithmic_flops,"
         "arithmetic_intensity_flop_per_byte,blocks,threads,result,result_bits,"
         "timing_status\n";
  write_env(out, env);
  out << ',' << name_of(o.run_mode) << ',' << spec.id << ',' << name_of(o.one) << ",float32,"
      << (fp64(o.one) ? "float64" : "float32") << ',' << (raw(o.one) ? "raw" : "accessor") << ','
      << in.count << ',' << 8.0 * static_cast<double>(in.count) << ','
      << 2.0 * static_cast<double>(in.count) << ",0.25," << sm_count << ",256,"
      << std::setprecision(21) << static_cast<long double>(got) << ',' << bits_of(got)
      << ",profiler_contaminated\n";
}

} // namespace

int main(int argc, char **argv) {
  try {
    bool help = false;
    const options o = parse(argc, argv, help);
    if (help) {
      usage(argv[0]);
      return 0;
    }
    int device = 0;
    cuda_check(cudaGetDevice(&device), "cudaGetDevice");
    const environment env = probe(device);
    aut_workspace *ws = nullptr;
    aut_check(aut_workspace_create(device, &ws), "aut_workspace_create");
    cudaStream_t s = nullptr;
    cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
    std::ofstream file;
    std::ostream *out = &std::cout;
    if (o.output != "-") {
      file.open(o.output);
      if (!file) throw std::runtime_error("cannot open output: " + o.output);
      out = &file;
    }
    if (o.run_mode == mode::performance) performance(o, env, ws, s, *out);
    else if (o.run_mode == mode::accuracy) accuracy(o, env, ws, s, *out);
    else profile(o, env, ws, s, *out);
    cudaStreamDestroy(s);
    aut_workspace_destroy(ws);
    return 0;
  } catch (const std::exception &e) {
    std::cerr << "error: " << e.what() << '\n';
    return 1;
  }
}
