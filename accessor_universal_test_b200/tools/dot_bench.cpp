// dot_bench -- raw FP32/FP64 DOT: cuBLAS Sdot/Ddot next to libautdot.
//
// Flags, datasets, timing loop and CSV schema of the reference's
// src/dot_bench.cu (options :173-189, parser :242-340, generators :361-424,
// statistics :468-506, accuracy :532-577, header :633-641, row :643-671,
// run_one :673-749).  Operations: sdot / ddot (cuBLAS, device pointer mode,
// as in the reference), aut (the fused DOT: FP32 storage with FP32 and with
// FP64 accumulation, FP64 storage with FP64 accumulation), both (= sdot+ddot)
// and all (default).
#include <autdot.h>

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <ctime>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <limits>
#include <numeric>
#include <sstream>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

namespace {

void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
void blas_check(cublasStatus_t s, const char *what) {
  if (s != CUBLAS_STATUS_SUCCESS)
    throw std::runtime_error(std::string(what) + " failed: " + std::to_string(s));
}
void aut_check(aut_status s, const char *what) {
  if (s != AUT_OK) throw std::runtime_error(std::string(what) + ": " + aut_last_error());
}

enum class mode { performance, accuracy, profile };
enum class dataset { positive, signed_uniform, cancellation, dynamic_range };

struct options {
  mode run_mode{mode::performance};
  bool sdot{true}, ddot{true}, aut{true};
  dataset data{dataset::signed_uniform};
  std::vector<int> powers{10, 16, 20, 23, 26, 27};
  int warmup{5};
  int samples{20};
  int iterations{0};
  double target_sample_ms{20.0};
  uint64_t seed{0x123456789abcdef0ULL};
  std::string output{"-"};
};

const char *mode_name(mode m) {
  return m == mode::performance ? "performance" : m == mode::accuracy ? "accuracy" : "profile";
}
const char *dataset_name(dataset d) {
  switch (d) {
  case dataset::positive: return "positive";
  case dataset::signed_uniform: return "signed";
  case dataset::cancellation: return "cancellation";
  case dataset::dynamic_range: return "dynamic";
  }
  return "unknown";
}

options parse(int argc, char **argv) {
  options o;
  bool powers_set = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto value = [&]() -> std::string {
      if (++i >= argc) throw std::runtime_error("missing value after " + a);
      return argv[i];
    };
    if (a == "--mode") {
      const auto v = value();
      o.run_mode = v == "accuracy" ? mode::accuracy : v == "profile" ? mode::profile
                   : v == "performance" ? mode::performance
                                        : throw std::runtime_error("unknown mode: " + v);
    } else if (a == "--operation") {
      const auto v = value();
      o.sdot = v == "sdot" || v == "both" || v == "all";
      o.ddot = v == "ddot" || v == "both" || v == "all";
      o.aut = v == "aut" || v == "all";
      if (!o.sdot && !o.ddot && !o.aut) throw std::runtime_error("unknown operation: " + v);
    } else if (a == "--dataset") {
      const auto v = value();
      o.data = v == "positive" ? dataset::positive : v == "signed" ? dataset::signed_uniform
               : v == "cancellation" ? dataset::cancellation
               : v == "dynamic" ? dataset::dynamic_range
                                : throw std::runtime_error("unknown dataset: " + v);
    } else if (a == "--powers") {
      o.powers.clear();
      std::stringstream ss(value());
      std::string t;
      while (std::getline(ss, t, ',')) o.powers.push_back(std::stoi(t));
      powers_set = true;
    } else if (a == "--n") {
      const uint64_t n = std::stoull(value(), nullptr, 0);
      if (n == 0 || (n & (n - 1)) != 0) throw std::runtime_error("--n must be a nonzero power of two");
      int p = 0;
      for (uint64_t v = n; v > 1; v >>= 1) ++p;
      o.powers = {p};
      powers_set = true;
    } else if (a == "--warmup") o.warmup = std::stoi(value());
    else if (a == "--samples") o.samples = std::stoi(value());
    else if (a == "--iterations") o.iterations = std::stoi(value());
    else if (a == "--target-sample-ms") o.target_sample_ms = std::stod(value());
    else if (a == "--seed") o.seed = std::stoull(value(), nullptr, 0);
    else if (a == "--output") o.output = value();
    else if (a == "--help" || a == "-h") {
      std::cout << "dot_bench --mode performance|accuracy|profile --operation "
                   "sdot|ddot|both|aut|all --dataset positive|signed|cancellation|dynamic "
                   "--powers P1,P2 | --n N --warmup N --samples N --iterations N "
                   "--target-sample-ms X --seed N --output PATH\n";
      std::exit(0);
    } else throw std::runtime_error("unknown argument: " + a);
  }
  if (!powers_set && o.run_mode == mode::accuracy) o.powers = {10, 16, 20};
  if (!powers_set && o.run_mode == mode::profile) o.powers = {27};
  for (int p : o.powers)
    if (p < 0 || p > 30) throw std::runtime_error("powers must be in [0, 30]");
  return o;
}

// The reference's dot_bench generators (src/dot_bench.cu:361-424).
uint64_t splitmix64(uint64_t v) {
  v += 0x9e3779b97f4a7c15ULL;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ULL;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebULL;
  return v ^ (v >> 31);
}
template <typename T> T positive_unit(uint64_t bits) {
  if constexpr (std::is_same_v<T, float>)
    return static_cast<float>(static_cast<uint32_t>(bits >> 40) + 1u) * 0x1p-24f;
  else
    return static_cast<double>((bits >> 11) + 1ULL) * 0x1p-53;
}
template <typename T> T signed_unit(uint64_t bits) {
  if constexpr (std::is_same_v<T, float>)
    return static_cast<float>(static_cast<int32_t>(static_cast<uint32_t>(bits >> 41)) - (1 << 22)) *
           0x1p-22f;
  else
    return static_cast<double>(static_cast<int64_t>(bits >> 12) - (1LL << 51)) * 0x1p-51;
}
template <typename T> T sample_value(uint64_t i, uint64_t seed, dataset d, int vid) {
  const uint64_t lane = seed ^ (0xd1b54a32d192ed03ULL * static_cast<uint64_t>(vid + 1));
  const uint64_t bits = splitmix64(i ^ lane);
  if (d == dataset::positive) return positive_unit<T>(bits);
  if (d == dataset::signed_uniform) return signed_unit<T>(bits);
  if (d == dataset::cancellation) {
    if (vid == 0) return T{1};
    const T m = positive_unit<T>(splitmix64((i / 2) ^ lane));
    return (i & 1ULL) == 0 ? m : -m * (T{1} - static_cast<T>(0x1p-10));
  }
  const int e = static_cast<int>((bits >> 1) % 41ULL) - 20;
  return ((bits & 1ULL) ? T{-1} : T{1}) * std::ldexp(positive_unit<T>(bits), e);
}

struct stats {
  double min{}, median{}, p10{}, p90{}, mean{}, cv{};
};
double pct(const std::vector<double> &s, double p) {
  if (s.size() == 1) return s[0];
  const double pos = p * static_cast<double>(s.size() - 1);
  const size_t lo = static_cast<size_t>(pos);
  const size_t hi = std::min(lo + 1, s.size() - 1);
  return s[lo] + (pos - static_cast<double>(lo)) * (s[hi] - s[lo]);
}
stats summarize(std::vector<double> s) {
  std::sort(s.begin(), s.end());
  stats r;
  r.min = s.front();
  r.median = pct(s, 0.5);
  r.p10 = pct(s, 0.1);
  r.p90 = pct(s, 0.9);
  r.mean = std::accumulate(s.begin(), s.end(), 0.0) / s.size();
  double var = 0;
  for (double v : s) var += (v - r.mean) * (v - r.mean);
  var /= s.size();
  r.cv = r.mean == 0 ? 0 : std::sqrt(var) / r.mean;
  return r;
}

// Neumaier-compensated long double sum (src/dot_bench.cu:532-549).
struct comp_sum {
  long double sum{}, corr{};
  void add(long double v) {
    const long double u = sum + v;
    if (std::fabs(sum) >= std::fabs(v)) corr += (sum - u) + v;
    else corr += (v - u) + sum;
    sum = u;
  }
  long double value() const { return sum + corr; }
};

struct accuracy {
  long double reference = NAN, sum_abs = NAN, abs_err = NAN, rel_err = NAN, norm_err = NAN,
              cond = NAN;
};

template <typename T>
accuracy compute_accuracy(const std::vector<T> &x, const std::vector<T> &y, double computed) {
  comp_sum ref, sabs;
  for (size_t i = 0; i < x.size(); ++i) {
    const long double p = static_cast<long double>(x[i]) * static_cast<long double>(y[i]);
    ref.add(p);
    sabs.add(std::fabs(p));
  }
  accuracy a;
  a.reference = ref.value();
  a.sum_abs = sabs.value();
  a.abs_err = std::fabs(static_cast<long double>(computed) - a.reference);
  if (a.reference != 0.0L) {
    a.rel_err = a.abs_err / std::fabs(a.reference);
    a.cond = a.sum_abs / std::fabs(a.reference);
  }
  if (a.sum_abs != 0.0L) a.norm_err = a.abs_err / a.sum_abs;
  return a;
}

struct env {
  std::string gpu;
  int major{}, minor{}, runtime{}, driver{}, cublas{};
};

std::string csv_escape(const std::string &v) {
  if (v.find_first_of(",\"\n") == std::string::npos) return v;
  std::string e{"\""};
  for (char c : v) e += c == '"' ? std::string("\"\"") : std::string(1, c);
  return e + '"';
}

} // namespace

int main(int argc, char **argv) {
  try {
    const options o = parse(argc, argv);
    cudaStream_t stream;
    cuda_check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
    cublasHandle_t handle;
    blas_check(cublasCreate(&handle), "cublasCreate");
    blas_check(cublasSetStream(handle, stream), "cublasSetStream");
    blas_check(cublasSetPointerMode(handle, CUBLAS_POINTER_MODE_DEVICE), "pointer mode");
    aut_workspace *ws = nullptr;
    aut_check(aut_workspace_create(0, &ws), "aut_workspace_create");

    env e;
    cudaDeviceProp prop{};
    cuda_check(cudaGetDeviceProperties(&prop, 0), "props");
    e.gpu = prop.name;
    e.major = prop.major;
    e.minor = prop.minor;
    cudaRuntimeGetVersion(&e.runtime);
    cudaDriverGetVersion(&e.driver);
    cublasGetVersion(handle, &e.cublas);

    std::ofstream file;
    std::ostream *out = &std::cout;
    if (o.output != "-") {
      file.open(o.output);
      if (!file) throw std::runtime_error("could not open output file: " + o.output);
      out = &file;
    }
    *out << "gpu,compute_capability,cuda_runtime,cuda_driver,cublas_version,"
            "mode,dataset,operation,input_type,n,algorithmic_bytes,"
            "algorithmic_flops,arithmetic_intensity_flop_per_byte,iterations,"
            "samples,min_ms,median_ms,p10_ms,p90_ms,coefficient_of_variation,"
            "giga_elements_per_s,algorithmic_gb_per_s,gflop_per_s,result,"
            "reference,absolute_error,relative_error,normalized_error,"
            "dot_condition_number\n";

    cudaEvent_t a, b;
    cuda_check(cudaEventCreate(&a), "event");
    cuda_check(cudaEventCreate(&b), "event");

    auto run = [&](auto tag, size_t n, const std::string &op, auto launch, auto read_result,
                   const auto &hx, const auto &hy) {
      using T = decltype(tag);
      for (int w = 0; w < o.warmup; ++w) launch();
      cuda_check(cudaStreamSynchronize(stream), "warmup");
      int iterations = o.iterations;
      std::vector<double> times;
      auto elapsed = [&](int iters) {
        cuda_check(cudaEventRecord(a, stream), "record");
        for (int k = 0; k < iters; ++k) launch();
        cuda_check(cudaEventRecord(b, stream), "record");
        cuda_check(cudaEventSynchronize(b), "sync");
        float ms = 0;
        cuda_check(cudaEventElapsedTime(&ms, a, b), "elapsed");
        return static_cast<double>(ms);
      };
      stats st{};
      if (o.run_mode == mode::profile) {
        launch();
        cuda_check(cudaStreamSynchronize(stream), "profile");
        iterations = 1;
        const double nan = std::numeric_limits<double>::quiet_NaN();
        st = {nan, nan, nan, nan, nan, nan};
      } else {
        if (iterations == 0) {
          const double cal = elapsed(1);
          iterations = std::clamp(static_cast<int>(std::ceil(o.target_sample_ms / std::max(0.001, cal))), 1, 100000);
        }
        for (int s = 0; s < o.samples; ++s) times.push_back(elapsed(iterations) / iterations);
        st = summarize(times);
      }
      const double result = read_result();
      accuracy acc;
      if (o.run_mode == mode::accuracy) acc = compute_accuracy(hx, hy, result);
      const double bytes = 2.0 * n * sizeof(T), flops = 2.0 * n, sec = st.median * 1e-3;
      *out << csv_escape(e.gpu) << ',' << e.major << '.' << e.minor << ',' << e.runtime << ','
           << e.driver << ',' << e.cublas << ',' << mode_name(o.run_mode) << ','
           << dataset_name(o.data) << ',' << op << ','
           << (std::is_same_v<T, float> ? "float32" : "float64") << ',' << n << ','
           << static_cast<uint64_t>(bytes) << ',' << std::setprecision(17) << flops << ','
           << flops / bytes << ',' << iterations << ',' << (o.run_mode == mode::profile ? 1 : o.samples)
           << ',' << st.min << ',' << st.median << ',' << st.p10 << ',' << st.p90 << ','
           << st.cv << ',' << n / sec / 1e9 << ',' << bytes / sec / 1e9 << ','
           << flops / sec / 1e9 << ',' << std::setprecision(21) << result << ','
           << acc.reference << ',' << acc.abs_err << ',' << acc.rel_err << ',' << acc.norm_err
           << ',' << acc.cond << '\n';
      std::cerr << op << " N=" << n << " median=" << st.median << " ms\n";
    };

    for (int power : o.powers) {
      const size_t n = size_t{1} << power;
      for (int fp64 = 0; fp64 < 2; ++fp64) {
        auto body = [&](auto tag) {
          using T = decltype(tag);
          std::vector<T> hx(n), hy(n);
          for (size_t i = 0; i < n; ++i) {
            hx[i] = sample_value<T>(i, o.seed, o.data, 0);
            hy[i] = sample_value<T>(i, o.seed, o.data, 1);
          }
          T *dx, *dy;
          double *dres;
          cuda_check(cudaMalloc(&dx, n * sizeof(T)), "malloc");
          cuda_check(cudaMalloc(&dy, n * sizeof(T)), "malloc");
          cuda_check(cudaMalloc(&dres, 2 * sizeof(double)), "malloc");
          cuda_check(cudaMemcpy(dx, hx.data(), n * sizeof(T), cudaMemcpyHostToDevice), "h2d");
          cuda_check(cudaMemcpy(dy, hy.data(), n * sizeof(T), cudaMemcpyHostToDevice), "h2d");
          const bool want_blas = std::is_same_v<T, float> ? o.sdot : o.ddot;
          if (want_blas) {
            if (n > static_cast<size_t>(std::numeric_limits<int>::max()))
              throw std::runtime_error("vector size exceeds the cuBLAS 32-bit API");
            T *dblas = reinterpret_cast<T *>(dres + 1);
            auto launch = [&] {
              if constexpr (std::is_same_v<T, float>)
                blas_check(cublasSdot(handle, static_cast<int>(n), dx, 1, dy, 1, dblas), "cublasSdot");
              else
                blas_check(cublasDdot(handle, static_cast<int>(n), dx, 1, dy, 1, dblas), "cublasDdot");
            };
            auto read = [&] {  // cuBLAS writes its own type T
              T v{};
              cuda_check(cudaMemcpyAsync(&v, dblas, sizeof v, cudaMemcpyDeviceToHost, stream), "copy");
              cuda_check(cudaStreamSynchronize(stream), "sync");
              return static_cast<double>(v);
            };
            run(T{}, n, std::is_same_v<T, float> ? "cublasSdot" : "cublasDdot", launch, read, hx, hy);
          }
          if (o.aut) {
            const int32_t fid = std::is_same_v<T, float> ? AUT_FMT_FP32 : AUT_FMT_FP64;
            auto read = [&] {
              double v = 0;
              cuda_check(cudaMemcpyAsync(&v, dres, sizeof v, cudaMemcpyDeviceToHost, stream), "copy");
              cuda_check(cudaStreamSynchronize(stream), "sync");
              return v;
            };
            for (int32_t accum : {AUT_ACCUM_FP32, AUT_ACCUM_FP64}) {
              if (!aut_dot_supported(fid, AUT_LAYOUT_DENSE, accum)) continue;
              const std::string op = accum == AUT_ACCUM_FP32 ? "aut_dot_acc32" : "aut_dot_acc64";
              run(T{}, n, op,
                  [&] { aut_check(aut_dot(ws, fid, AUT_LAYOUT_DENSE, accum, dx, dy, n, dres, stream), "aut_dot"); },
                  read, hx, hy);
            }
          }
          cudaFree(dx);
          cudaFree(dy);
          cudaFree(dres);
        };
        if (fp64) body(double{});
        else body(float{});
      }
      out->flush();
    }
    aut_workspace_destroy(ws);
    cublasDestroy(handle);
    cudaStreamDestroy(stream);
    return 0;
  } catch (const std::exception &ex) {
    std::cerr << "error: " << ex.what() << '\n';
    return 1;
  }
}
