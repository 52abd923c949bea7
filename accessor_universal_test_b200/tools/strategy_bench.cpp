// strategy_bench -- the reference's strategy benchmarks on libautdot.
//
// Flags and CSV schemas of src/bitwidth_strategy_bench.cu (options :76-153,
// header :448-453) and src/lns_strategy_bench.cu (options :80-160, header
// :626-633), so the reference's validators and summarisers read the output
// unchanged.  Differences: formats are chosen at run time (--formats) instead
// of one binary per width, the access strategies are this library's
// (scalar / thread_packet = LDG / tma_bulk = TMA), data come from the seeded
// generators of aut_generate (uniform_0_1: (0,1]; normal_0_1: Irwin-Hall)
// instead of cuRAND.  GEMV rows (kernel "gemv", --gemv-powers / --gemv-rows,
// src/bitwidth_strategy_bench.cu:653-684) time aut_gemv over the same
// strategies and decoders.  The scalar rows (one value per thread, AUTO
// decoder) carry the decoder names the reference's smoke validators take as
// their baseline: "generic" (bitwidth) and "reference_exp2" (LNS).
#include <autdot.h>

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <ctime>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <set>
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
  if (s != AUT_OK)
    throw std::runtime_error(std::string(what) + ": " + aut_last_error());
}

std::vector<std::string> split(const std::string &text) {
  std::vector<std::string> out;
  std::stringstream ss(text);
  std::string tok;
  while (std::getline(ss, tok, ','))
    if (!tok.empty()) out.push_back(tok);
  return out;
}

struct options {
  std::string family{"bitwidth"};
  std::vector<std::string> formats;
  std::string mode{"screen"};
  std::vector<int> dot_powers{24};
  std::vector<int> gemv_powers{14};
  uint64_t gemv_rows{1024};
  std::vector<std::string> distributions{"uniform_0_1", "normal_0_1"};
  std::vector<std::string> accums{"fp32", "fp64"};
  int warmup{5};
  int samples{3};
  double target_sample_ms{10.0};
  uint64_t seed{0x243f6a8885a308d3ull};
  std::string output;
  std::set<std::string> variants;
};

options parse(int argc, char **argv) {
  options o;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto value = [&]() -> std::string {
      if (++i >= argc) throw std::runtime_error("missing value after " + a);
      return argv[i];
    };
    if (a == "--family") o.family = value();
    else if (a == "--formats") o.formats = split(value());
    else if (a == "--mode") o.mode = value();
    else if (a == "--dot-powers") {
      o.dot_powers.clear();
      for (auto &t : split(value())) o.dot_powers.push_back(std::stoi(t));
    } else if (a == "--gemv-powers") {
      o.gemv_powers.clear();
      for (auto &t : split(value())) o.gemv_powers.push_back(std::stoi(t));
    } else if (a == "--gemv-rows") o.gemv_rows = std::stoull(value());
    else if (a == "--distributions") o.distributions = split(value());
    else if (a == "--accums") o.accums = split(value());
    else if (a == "--warmup") o.warmup = std::stoi(value());
    else if (a == "--samples") o.samples = std::stoi(value());
    else if (a == "--target-sample-ms") o.target_sample_ms = std::stod(value());
    else if (a == "--seed") o.seed = std::stoull(value(), nullptr, 0);
    else if (a == "--output") o.output = value();
    else if (a == "--variants") for (auto &t : split(value())) o.variants.insert(t);
    else if (a == "--variant-file") {
      std::ifstream in(value());
      if (!in) throw std::runtime_error("cannot open variant file");
      std::string line;
      while (std::getline(in, line))
        if (!line.empty() && line[0] != '#') o.variants.insert(line);
    } else if (a == "--help" || a == "-h") {
      std::cout << "strategy_bench --family bitwidth|lns --formats e2m3,e8m0,... "
                   "--mode smoke|screen|full --dot-powers 24 --gemv-powers 14 "
                   "--gemv-rows 1024 --distributions "
                   "uniform_0_1,normal_0_1 --accums fp32,fp64 --warmup N --samples N "
                   "--target-sample-ms X --seed N --output PATH [--variants a,b] "
                   "[--variant-file PATH]\n";
      std::exit(0);
    } else throw std::runtime_error("unknown option: " + a);
  }
  if (o.family != "bitwidth" && o.family != "lns")
    throw std::runtime_error("--family must be bitwidth or lns");
  if (o.formats.empty())
    o.formats = o.family == "lns" ? std::vector<std::string>{"lns8_r3", "lns16_r11"}
                                  : std::vector<std::string>{"e2m3", "e8m0", "e8m1", "e8m3",
                                                             "e8m5", "bf16_e8m7", "e8m15"};
  if (o.output.empty())
    o.output = o.family == "lns" ? "lns_timing_samples.csv" : "timing_samples.csv";
  if (o.mode == "smoke") {  // the reference's smoke overrides
    o.dot_powers = {12};
    o.gemv_powers = {8};
    o.gemv_rows = 32;
    o.warmup = 1;
    o.samples = 1;
    o.target_sample_ms = 0.0;
  }
  return o;
}

std::string utc_now() {
  const auto t = std::chrono::system_clock::to_time_t(std::chrono::system_clock::now());
  std::tm utc{};
  gmtime_r(&t, &utc);
  std::ostringstream s;
  s << std::put_time(&utc, "%Y-%m-%dT%H:%M:%SZ");
  return s.str();
}

struct device_buffer {
  void *p = nullptr;
  explicit device_buffer(size_t bytes) { cuda_check(cudaMalloc(&p, bytes < 16 ? 16 : bytes), "cudaMalloc"); }
  ~device_buffer() { cudaFree(p); }
  device_buffer(const device_buffer &) = delete;
  device_buffer &operator=(const device_buffer &) = delete;
};

int gcd_int(int a, int b) { return b == 0 ? a : gcd_int(b, a % b); }

struct access {
  const char *name;     // access_method column
  int32_t strategy;
  const char *redistribution;
};

// The decoders this library has for a format and accumulator, with the
// reference's decoder_kind / multiply_kind names (lns_decoder_strategies.cuh:19-36).
struct decoder_choice {
  int32_t id;
  const char *name;
  const char *multiply;  // LNS only
  int table_bytes;       // shared-memory table per block
};

std::vector<decoder_choice> decoders_for(const std::string &fmt, int32_t accum) {
  const int t = accum == AUT_ACCUM_FP64 ? 8 : 4;
  static const std::set<std::string> fused = {"fp32", "fp64", "e2m3", "e8m0", "e8m1",
                                              "e8m3", "e8m5", "bf16_e8m7", "e8m15",
                                              "lns8_r3", "lns16_r11"};
  if (!fused.count(fmt)) {  // the generic DOT (runtime format switch)
    const int32_t fid = aut_format_id(fmt.c_str());
    int32_t family = 0, bits = 0, e = 0, fin = 0;
    aut_format_info(fid, &family, &bits, &e, &fin);
    if (bits <= 8)  // table decode (every family), and the runtime shift for bit formats
      return family == AUT_FAMILY_LNS
                 ? std::vector<decoder_choice>{{AUT_DECODER_FULL_LUT, "full_lut_shared",
                                                "ordinary", (1 << bits) * 32 * t}}
                 : std::vector<decoder_choice>{{AUT_DECODER_FULL_LUT, "full_lut_shared",
                                                "ordinary", (1 << bits) * 32 * t},
                                               {AUT_DECODER_DIRECT, "direct_shift", "ordinary", 0}};
    if (family == AUT_FAMILY_LNS) {
      const int bytes = (1 << bits) * t;
      return {{AUT_DECODER_AUTO, bytes <= 32 * 1024 ? "full_lut_shared" : "full_lut_global",
               "ordinary", bytes}};
    }
    return {{AUT_DECODER_AUTO, "direct_shift", "ordinary", 0}};  // runtime E/M/bias
  }
  if (fmt == "lns8_r3")
    return {{AUT_DECODER_FULL_LUT, "full_lut_shared", "ordinary", 256 * 32 * t},
            {AUT_DECODER_FUSED_SUM_LUT, "fused_sum_lut_shared", "fused", 256 * 32 * t},
            {AUT_DECODER_EX2_APPROX, "ex2_approx", "fused", 0}};
  if (fmt == "lns16_r11") {
    std::vector<decoder_choice> d;
    if (accum == AUT_ACCUM_FP32)
      d.push_back({AUT_DECODER_FULL_LUT, "full_lut_shared", "ordinary", 32768 * 4});
    d.push_back({AUT_DECODER_FRACTION_LUT, "fraction_lut_shared", "ordinary", 2048 * t});
    d.push_back({AUT_DECODER_FRACTION_LUT_FUSED, "fraction_lut_shared", "fused", 2048 * t});
    d.push_back({AUT_DECODER_EX2_APPROX, "ex2_approx", "fused", 0});
    return d;
  }
  if (fmt == "e2m3")
    return {{AUT_DECODER_DIRECT, "native_packed", "ordinary", 0},
            {AUT_DECODER_FULL_LUT, "full_lut_shared", "ordinary", 64 * 32 * t}};
  if (fmt == "e8m0" || fmt == "e8m1" || fmt == "e8m3" || fmt == "e8m5") {
    const int32_t fid = aut_format_id(fmt.c_str());
    int32_t family = 0, bits = 0, e = 0, fin = 0;
    aut_format_info(fid, &family, &bits, &e, &fin);
    std::vector<decoder_choice> d = {{AUT_DECODER_DIRECT, "direct_shift", "ordinary", 0},
                                     {AUT_DECODER_FULL_LUT, "full_lut_shared", "ordinary",
                                      (1 << bits) * 4}};
    if (bits > 9) {  // the partial tables need mantissa bits
      d.push_back({AUT_DECODER_PREFIX_LUT, "prefix_lut_shared", "ordinary", 512 * 4});
      d.push_back({AUT_DECODER_SUBNORMAL_LUT, "subnormal_lut_shared", "ordinary",
                   (1 << (bits - 9)) * 4});
    }
    return d;
  }
  return {{AUT_DECODER_DIRECT, "direct_shift", "ordinary", 0}};
}

// The cooperative loader's chunk (cooperative_geometry of
// include/aut/bitwidth.hpp, for a runtime width).
struct coop_geometry {
  int values, words, consumers;
};
coop_geometry coop_geometry_of(int bits) {
  const int g = gcd_int(bits, 32);
  coop_geometry c{32 / g, bits / g, 0};
  int above = 1;
  while (above <= c.words) above *= 2;
  c.consumers = std::max({4, above, c.values / 4});
  c.consumers = std::min(c.consumers, c.values);
  return c;
}

} // namespace

int main(int argc, char **argv) {
  try {
    const options o = parse(argc, argv);
    cudaDeviceProp prop{};
    cuda_check(cudaGetDeviceProperties(&prop, 0), "cudaGetDeviceProperties");
    aut_workspace *ws = nullptr;
    aut_check(aut_workspace_create(0, &ws), "aut_workspace_create");
    std::cout << "Strategy benchmark (" << o.family << "): GPU " << prop.name << " (sm_"
              << prop.major << prop.minor << ")\n";

    std::ifstream existing(o.output, std::ios::binary | std::ios::ate);
    const bool header = !existing || existing.tellg() == 0;
    existing.close();
    std::ofstream csv(o.output, std::ios::app);
    if (!csv) throw std::runtime_error("cannot open output: " + o.output);
    if (header) {
      if (o.family == "lns")
        csv << "timestamp,gpu,mode,distribution,kernel,number_family,format,bits,"
               "log_integer_bits,log_fraction_bits,arithmetic_type,multiply_method,"
               "storage_layout,access_method,packet_values,load_word_bits,loader_threads,"
               "consumer_threads,values_per_consumer,redistribution,decoder,strategy_id,"
               "N,M,rows,logical_input_bytes,physical_input_bytes,table_bytes,blocks,"
               "threads,warmup,sample,iterations,total_ms,mean_ms,result,valid\n";
      else
        csv << "timestamp,gpu,mode,distribution,kernel,format,bits,exponent_bits,"
               "mantissa_bits,arithmetic_type,storage_layout,access_method,packet_values,"
               "load_word_bits,loader_threads,consumer_threads,values_per_consumer,"
               "redistribution,decoder,strategy_id,N,M,rows,logical_input_bytes,"
               "physical_input_bytes,table_bytes,blocks,threads,warmup,sample,iterations,"
               "total_ms,mean_ms,result,valid\n";
    }
    const std::string stamp = utc_now();
    int32_t sm = 0, max_blocks = 0;
    aut_workspace_info(ws, &sm, &max_blocks);

    cudaEvent_t start, stop;
    cuda_check(cudaEventCreate(&start), "event");
    cuda_check(cudaEventCreate(&stop), "event");
    double *d_result = nullptr;
    cuda_check(cudaMalloc(&d_result, sizeof(double)), "cudaMalloc");

    const access accesses[] = {{"scalar", AUT_STRATEGY_SCALAR, "none"},
                               {"thread_packet", AUT_STRATEGY_LDG, "none"},
                               {"tma_bulk", AUT_STRATEGY_TMA, "tma_bulk_shared"},
                               {"cooperative_shuffle", AUT_STRATEGY_COOPERATIVE,
                                "warp_shuffle"}};
    const int max_power = *std::max_element(o.dot_powers.begin(), o.dot_powers.end());
    uint64_t max_n = uint64_t{1} << max_power;
    for (int p : o.gemv_powers)
      max_n = std::max(max_n, (o.gemv_rows + 1) << p);
    device_buffer values(max_n * sizeof(double));
    device_buffer gemv_out(o.gemv_rows * sizeof(double));

    // Times `launch` (warm-up, a pilot to size samples of target_sample_ms,
    // then `samples` samples) and returns (iterations, per-sample ms).
    auto measure = [&](const auto &launch) {
      auto timed = [&](int iters) {
        cuda_check(cudaEventRecord(start), "record");
        for (int k = 0; k < iters; ++k) launch();
        cuda_check(cudaEventRecord(stop), "record");
        cuda_check(cudaEventSynchronize(stop), "sync");
        float ms = 0.f;
        cuda_check(cudaEventElapsedTime(&ms, start, stop), "elapsed");
        return static_cast<double>(ms);
      };
      for (int w = 0; w < o.warmup; ++w) launch();
      cuda_check(cudaDeviceSynchronize(), "warmup");
      const double pilot = timed(1);
      int iterations = 1;
      if (o.target_sample_ms > 0 && pilot > 0)
        iterations = std::clamp(static_cast<int>(std::ceil(o.target_sample_ms / pilot)), 1, 10000);
      std::vector<double> times;
      for (int k = 0; k < o.samples; ++k) times.push_back(timed(iterations));
      return std::make_pair(iterations, times);
    };

    for (size_t d = 0; d < o.distributions.size(); ++d) {
      const std::string &dist = o.distributions[d];
      const int32_t kind = dist == "uniform_0_1"  ? AUT_GEN_POSITIVE_UNIT_F64
                           : dist == "normal_0_1" ? AUT_GEN_NORMAL
                                                  : -1;
      if (kind < 0) throw std::runtime_error("unsupported distribution: " + dist);
      const uint64_t seed = o.seed + d * 0x9e3779b97f4a7c15ull;
      std::cout << dist << "\n";
      for (const auto &name : o.formats) {
        const int32_t fid = aut_format_id(name.c_str());
        if (fid < 0) throw std::runtime_error("unknown format: " + name);
        int32_t family = 0, bits = 0, ebits = 0, finite = 0;
        aut_format_info(fid, &family, &bits, &ebits, &finite);
        aut_check(aut_workspace_prepare(ws, fid), "aut_workspace_prepare");
        auto encode = [&](uint64_t vector_id, uint64_t n, int32_t layout, void *dst) {
          aut_check(aut_generate(kind, seed, vector_id, 0, n, static_cast<double *>(values.p), nullptr),
                    "generate");
          aut_check(aut_encode(ws, fid, layout, static_cast<double *>(values.p), n, dst, nullptr),
                    "encode");
        };
        for (const auto &acc_name : o.accums) {
          const int32_t accum = acc_name == "fp64" ? AUT_ACCUM_FP64 : AUT_ACCUM_FP32;
          std::cout << "  " << name << " -> " << acc_name << "\n";
          for (int32_t layout : {AUT_LAYOUT_DENSE, AUT_LAYOUT_PADDED}) {
            if (!aut_dot_supported(fid, layout, accum)) continue;
            const int stride = layout == AUT_LAYOUT_DENSE ? bits
                               : bits <= 8 ? 8 : bits <= 16 ? 16 : 32;
            auto physical_bytes = [&](uint64_t count) {
              return layout == AUT_LAYOUT_DENSE ? (count * bits + 7) / 8 : count * (stride / 8);
            };
            // One CSV row per sample (the reference's schema).
            auto emit = [&](const char *kernel, const access &ac, const decoder_choice &dc,
                            int packet, const std::string &id, uint64_t n, uint64_t m,
                            uint64_t rows, double logical, uint64_t physical, uint64_t blocks,
                            int iterations, const std::vector<double> &times, double result,
                            int valid) {
              for (size_t k = 0; k < times.size(); ++k) {
                csv << stamp << ',' << prop.name << ',' << o.mode << ',' << dist << ','
                    << kernel << ',';
                if (o.family == "lns")
                  csv << "lns," << name << ',' << bits << ',' << (bits - 1 - ebits) << ','
                      << ebits << ',' << acc_name << ',' << dc.multiply << ',';
                else
                  csv << name << ',' << bits << ',' << ebits << ',' << (bits - 1 - ebits)
                      << ',' << acc_name << ',';
                // cooperative rows: chunk values, words (loader lanes),
                // consumer lanes and values per consumer of the geometry
                const bool coop = ac.strategy == AUT_STRATEGY_COOPERATIVE;
                const coop_geometry cg = coop_geometry_of(bits);
                csv << (layout == AUT_LAYOUT_DENSE ? "dense" : "padded") << ',' << ac.name
                    << ',' << packet << ',' << (layout == AUT_LAYOUT_DENSE ? 32 : stride) << ','
                    << (coop ? cg.words : 1) << ','
                    << (coop ? cg.consumers : ac.strategy == AUT_STRATEGY_TMA ? 256 : 1) << ','
                    << (coop ? cg.values / cg.consumers : packet)
                    << ',' << ac.redistribution << ',' << dc.name << ',' << id << ',' << n
                    << ',' << m << ',' << rows << ',' << logical << ',' << physical << ','
                    << dc.table_bytes << ',' << blocks << ",256," << o.warmup << ',' << k
                    << ',' << iterations << ',' << times[k] << ',' << times[k] / iterations
                    << ',' << std::setprecision(17) << result << std::setprecision(6) << ','
                    << valid << '\n';
              }
            };
            auto status_ok = [&] {
              uint32_t status = 0;
              aut_check(aut_workspace_status(ws, &status, 1), "status");
              return status == 0;
            };
            for (const access &ac : accesses) {
              const bool scalar = ac.strategy == AUT_STRATEGY_SCALAR;
              const int packet = scalar ? 1
                                 : ac.strategy == AUT_STRATEGY_COOPERATIVE
                                     ? coop_geometry_of(bits).values
                                 : ac.strategy == AUT_STRATEGY_LDG
                                     ? 128 * (stride / gcd_int(stride, 128)) / stride
                                     : (stride >= 24 ? 16 : 32);
              std::vector<decoder_choice> choices = decoders_for(name, accum);
              if (scalar) {
                // the validators' baseline row: one per format and accumulator
                decoder_choice base = choices.back();
                if (name == "lns16_r11") base = choices[accum == AUT_ACCUM_FP32 ? 1 : 0];
                base.id = AUT_DECODER_AUTO;
                base.name = o.family == "lns" ? "reference_exp2" : "generic";
                base.multiply = "ordinary";
                choices = {base};
              }
              for (const decoder_choice &dc : choices) {
                std::ostringstream id;
                if (o.family == "lns") id << dc.multiply << '/';
                id << (layout == AUT_LAYOUT_DENSE ? "dense" : "padded") << '/' << ac.name
                   << "/x" << packet << '/' << dc.name;
                const std::string qualified = name + "/" + acc_name + "/" + id.str();
                if (!o.variants.empty() && !o.variants.count(id.str()) &&
                    !o.variants.count(qualified))
                  continue;
                // formats without fused kernels take the per-value access only
                {
                  device_buffer probe(64);
                  const aut_status st = aut_dot_variant(ws, fid, layout, accum, ac.strategy,
                                                        dc.id, probe.p, probe.p, 0, d_result,
                                                        nullptr);
                  if (st == AUT_ERR_UNSUPPORTED) continue;
                  aut_check(st, "aut_dot_variant");
                }
                for (int power : o.dot_powers) {
                  const uint64_t n = uint64_t{1} << power;
                  device_buffer xs(aut_storage_bytes(fid, layout, n));
                  device_buffer ys(aut_storage_bytes(fid, layout, n));
                  encode(0, n, layout, xs.p);
                  encode(1, n, layout, ys.p);
                  cuda_check(cudaDeviceSynchronize(), "encode");
                  const auto [iterations, times] = measure([&] {
                    aut_check(aut_dot_variant(ws, fid, layout, accum, ac.strategy, dc.id, xs.p,
                                              ys.p, n, d_result, nullptr),
                              "aut_dot_variant");
                  });
                  double result = 0.0;
                  cuda_check(cudaMemcpy(&result, d_result, sizeof result, cudaMemcpyDeviceToHost),
                             "copy");
                  const int valid = std::isfinite(result) && status_ok() ? 1 : 0;
                  emit("dot", ac, dc, packet, id.str(), n, 0, 1, 2.0 * n * bits / 8.0,
                       2 * physical_bytes(n), max_blocks, iterations, times, result, valid);
                }
                for (int power : o.gemv_powers) {
                  const uint64_t columns = uint64_t{1} << power;
                  const uint64_t rows = o.gemv_rows;
                  device_buffer ms(aut_storage_bytes(fid, layout, rows * columns));
                  device_buffer vs(aut_storage_bytes(fid, layout, columns));
                  encode(0, rows * columns, layout, ms.p);
                  encode(1, columns, layout, vs.p);
                  cuda_check(cudaDeviceSynchronize(), "encode");
                  double *out = static_cast<double *>(gemv_out.p);
                  const auto [iterations, times] = measure([&] {
                    aut_check(aut_gemv(ws, fid, layout, accum, ac.strategy, dc.id, ms.p, vs.p,
                                       rows, columns, out, nullptr),
                              "aut_gemv");
                  });
                  double first = 0.0;
                  cuda_check(cudaMemcpy(&first, out, sizeof first, cudaMemcpyDeviceToHost), "copy");
                  const int valid = std::isfinite(first) && status_ok() ? 1 : 0;
                  const uint64_t count = rows * columns + columns;
                  emit("gemv", ac, dc, packet, id.str(), columns, rows, rows,
                       static_cast<double>(count) * bits / 8.0, physical_bytes(count), rows,
                       iterations, times, first, valid);
                }
                if (o.mode == "smoke") std::cout << "    " << qualified << "\n";
              }
            }
          }
        }
      }
    }
    csv.flush();
    cudaFree(d_result);
    aut_workspace_destroy(ws);
    std::cout << "Wrote " << o.output << "\n";
    return 0;
  } catch (const std::exception &e) {
    std::cerr << "error: " << e.what() << "\n";
    return 1;
  }
}
