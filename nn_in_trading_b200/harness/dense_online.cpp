// dense_online: a C++ host that trains a dense network online (one sample per step) through the
// library's C ABI alone (include/nn_b200.h), issuing the kernel sequence of the reference's CNet for
// a stack of CNeuronBaseOCL layers:
//
//   forward      l = 1..L-1   FeedForward of layer l from layer l-1
//                             (CNeuronBaseOCL::feedForward, NeuroNet_Core.mqh:15686-15740)
//   output grad  layer L-1    CalcOutputGradient against the target
//                             (CNeuronBaseOCL::calcOutputGradients, NeuroNet_Core.mqh:15800-15837)
//   hidden grads l = L-2..0   CalcHiddenGradient of layer l from layer l+1
//                             (CNeuronBaseOCL::calcHiddenGradients, NeuroNet_Core.mqh:15744-15769)
//   updates      l = L-1..1   UpdateWeightsAdam of layer l-1's weights, then NormalizeWeights
//                             (CNeuronBaseOCL::updateInputWeights, NeuroNet_Core.mqh:15869-15984)
//
// The Adam rate of each update is bias-corrected on the host in double from the updating layer's
// step counter and passed as a float, as NeuroNet_Core.mqh:15903 does; the counter then advances.
// The NDRanges are the reference's: FeedForward and CalcHiddenGradient run (neurons, loc) work-items
// in (1, loc) groups with loc = min(ceil(n / 4), 256) over the n inputs they reduce.
//
// Every step writes the sample and its target to the device and reads the network's output back,
// as CNet::backPropOCL does to form its loss (NeuroNet_Core.mqh:13584-13599).
//
// Usage
//   dense_online --dir D --steps N [--device K]
//       D/net.txt: line 1 the layer sizes, line 2 the layer activations (NN_ACT_* values), both
//       comma-separated; D/w<l>.f32: the weights of layer l toward layer l+1, [next][n + 1] float32
//       with the bias last; D/x.f32 and D/t.f32: N samples and N targets.  Writes D/y.f32 (the
//       output of every step's forward pass) and D/w<l>.out.f32, D/m<l>.out.f32, D/v<l>.out.f32 (the
//       weights and Adam moments after the last step).
//   dense_online --synthetic --steps N [--device K]
//       240-500-500-3 (tanh, sigmoid, linear) with seeded uniform weights and inputs; prints one JSON
//       line with the steps per second measured around the whole loop on the host clock (device
//       work, launches and the per-step copies included).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "nn_b200.h"

namespace {

constexpr double kLR = 3.0e-4, kB1 = 0.9, kB2 = 0.999;  // NeuroNet_Definitions.mqh:38-46
constexpr int kMaxLocal = 256;                          // the local size the host reports to the layers

[[noreturn]] void die(const std::string &what) {
  std::fprintf(stderr, "dense_online: %s\n", what.c_str());
  std::exit(1);
}

int check(int rc, const char *call) {
  if (rc < 0) {
    char msg[512] = {0};
    nn_last_error(msg, (int)sizeof(msg));
    die(std::string(call) + " failed (" + std::to_string(rc) + "): " + msg);
  }
  return rc;
}
#define NN(call) check((call), #call)

std::vector<float> read_f32(const std::string &path, size_t count) {
  std::ifstream f(path, std::ios::binary);
  if (!f) die("cannot open " + path);
  std::vector<float> v(count);
  f.read(reinterpret_cast<char *>(v.data()), (std::streamsize)(count * sizeof(float)));
  if ((size_t)f.gcount() != count * sizeof(float)) die(path + ": expected " + std::to_string(count) + " floats");
  return v;
}

void write_f32(const std::string &path, const std::vector<float> &v) {
  std::ofstream f(path, std::ios::binary);
  if (!f) die("cannot write " + path);
  f.write(reinterpret_cast<const char *>(v.data()), (std::streamsize)(v.size() * sizeof(float)));
}

std::vector<int> parse_ints(const std::string &line) {
  std::vector<int> out;
  std::stringstream ss(line);
  std::string item;
  while (std::getline(ss, item, ',')) {
    if (item.empty()) continue;
    size_t used = 0;
    int v = 0;
    try {
      v = std::stoi(item, &used);
    } catch (const std::exception &) {
      used = 0;
    }
    if (used == 0 || item.find_first_not_of(" \t\r", used) != std::string::npos) die("not an integer: '" + item + "'");
    out.push_back(v);
  }
  return out;
}

// xorshift64*: uniform floats for the synthetic run
struct Rng {
  uint64_t s;
  explicit Rng(uint64_t seed) : s(seed ? seed : 1) {}
  double uniform() {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return (double)((s * 0x2545F4914F6CDD1DULL) >> 11) / 9007199254740992.0;
  }
  float range(double lo, double hi) { return (float)(lo + (hi - lo) * uniform()); }
};

// Bias-corrected Adam rate of update number t, in double, passed on as a float.
float adam_lt(int t) {
  return (float)(kLR * std::sqrt(1.0 - std::pow(kB2, t)) / (1.0 - std::pow(kB1, t)));
}

struct Layer {
  int neurons = 0, activation = NN_ACT_NONE, outputs = 0;
  int output = -1, gradient = -1, weights = -1, m = -1, v = -1;
  int t = 1;  // Adam step counter of the updates this layer runs on its input weights
};

class DenseNet {
 public:
  DenseNet(const std::vector<int> &sizes, const std::vector<int> &acts) {
    if (sizes.size() < 2 || sizes.size() != acts.size()) die("need at least two layers and one activation each");
    layers_.resize(sizes.size());
    for (size_t l = 0; l < sizes.size(); ++l) {
      Layer &L = layers_[l];
      L.neurons = sizes[l];
      L.activation = acts[l];
      L.outputs = l + 1 < sizes.size() ? sizes[l + 1] : 0;
      if (L.neurons <= 0) die("layer sizes must be positive");
      L.output = NN(nn_buffer_create(4LL * L.neurons));
      L.gradient = NN(nn_buffer_create(4LL * L.neurons));
      if (L.outputs) {
        const long long n = (long long)L.outputs * (L.neurons + 1);
        L.weights = NN(nn_buffer_create(4 * n));
        L.m = NN(nn_buffer_create(4 * n));  // created zero-filled
        L.v = NN(nn_buffer_create(4 * n));
      }
    }
    target_ = NN(nn_buffer_create(4LL * layers_.back().neurons));
    bind();
  }

  size_t size() const { return layers_.size(); }
  const Layer &layer(size_t l) const { return layers_[l]; }
  long long weight_count(size_t l) const {
    return (long long)layers_[l].outputs * (layers_[l].neurons + 1);
  }

  void set_weights(size_t l, const std::vector<float> &w) {
    if ((long long)w.size() != weight_count(l)) die("weight count mismatch");
    NN(nn_buffer_write(layers_[l].weights, w.data(), 0, (long long)w.size()));
  }

  std::vector<float> read(int handle, long long count) const {
    std::vector<float> v((size_t)count);
    NN(nn_buffer_read(handle, v.data(), 0, count));
    return v;
  }

  // One online step: the sample and its target in, the forward output back.
  void step(const float *x, const float *t, float *y) {
    const Layer &in = layers_.front(), &out = layers_.back();
    NN(nn_buffer_write(in.output, x, 0, in.neurons));
    NN(nn_buffer_write(target_, t, 0, out.neurons));
    for (const Exec &e : forward_) run(e);
    NN(nn_buffer_read(out.output, y, 0, out.neurons));  // blocking, like CBufferFloat::BufferRead
    for (const Exec &e : backward_) run(e);
    for (const Upd &u : updates_) {
      Layer &owner = layers_[u.owner];
      NN(nn_set_arg_float(u.adam.id, 6, adam_lt(owner.t)));
      ++owner.t;
      run(u.adam);
      run(u.normalize);
    }
  }

 private:
  struct Exec {
    int id, dims;
    unsigned g[2], l[2];
    bool local;
  };
  struct Upd {
    size_t owner;
    Exec adam, normalize;
  };

  int new_kernel(const char *name) {
    const int id = next_id_++;
    NN(nn_kernel_create(id, name));
    return id;
  }

  static int loc_for(int n) { return std::min((n + 3) / 4, kMaxLocal); }

  void run(const Exec &e) { NN(nn_execute(e.id, e.dims, nullptr, e.g, e.local ? e.l : nullptr)); }

  // Every kernel instance is bound once; executions only patch the Adam rate.
  void bind() {
    const size_t L = layers_.size();
    for (size_t l = 1; l < L; ++l) {
      const Layer &prev = layers_[l - 1], &cur = layers_[l];
      const int id = new_kernel("FeedForward");
      NN(nn_set_arg_buffer(id, 0, prev.weights));
      NN(nn_set_arg_buffer(id, 1, prev.output));
      NN(nn_set_arg_buffer(id, 2, cur.output));
      NN(nn_set_arg_int(id, 3, prev.neurons));
      NN(nn_set_arg_int(id, 4, cur.activation));
      NN(nn_set_arg_buffer(id, 5, cur.output));
      NN(nn_set_arg_int(id, 6, 0));
      const unsigned loc = (unsigned)loc_for(prev.neurons);
      forward_.push_back({id, 2, {(unsigned)cur.neurons, loc}, {1, loc}, true});
    }
    {
      const Layer &out = layers_.back();
      const int id = new_kernel("CalcOutputGradient");
      NN(nn_set_arg_buffer(id, 0, target_));
      NN(nn_set_arg_buffer(id, 1, out.output));
      NN(nn_set_arg_buffer(id, 2, out.gradient));
      NN(nn_set_arg_int(id, 3, out.activation));
      NN(nn_set_arg_float(id, 4, 1.0f));
      backward_.push_back({id, 1, {(unsigned)out.neurons, 0}, {0, 0}, false});
    }
    for (size_t l = L - 1; l-- > 0;) {
      const Layer &cur = layers_[l], &nxt = layers_[l + 1];
      const int id = new_kernel("CalcHiddenGradient");
      NN(nn_set_arg_buffer(id, 0, cur.weights));
      NN(nn_set_arg_buffer(id, 1, nxt.gradient));
      NN(nn_set_arg_buffer(id, 2, cur.output));
      NN(nn_set_arg_buffer(id, 3, cur.gradient));
      NN(nn_set_arg_int(id, 4, nxt.neurons));
      NN(nn_set_arg_int(id, 5, cur.activation));
      const unsigned loc = (unsigned)loc_for(nxt.neurons);
      backward_.push_back({id, 2, {(unsigned)cur.neurons, loc}, {1, loc}, true});
    }
    for (size_t l = L - 1; l >= 1; --l) {
      const Layer &prev = layers_[l - 1], &cur = layers_[l];
      const int ida = new_kernel("UpdateWeightsAdam");
      NN(nn_set_arg_buffer(ida, 0, prev.weights));
      NN(nn_set_arg_buffer(ida, 1, cur.gradient));
      NN(nn_set_arg_buffer(ida, 2, prev.output));
      NN(nn_set_arg_buffer(ida, 3, prev.m));
      NN(nn_set_arg_buffer(ida, 4, prev.v));
      NN(nn_set_arg_int(ida, 5, prev.neurons));
      NN(nn_set_arg_float(ida, 6, (float)kLR));
      NN(nn_set_arg_float(ida, 7, (float)kB1));
      NN(nn_set_arg_float(ida, 8, (float)kB2));
      const int idn = new_kernel("NormalizeWeights");
      NN(nn_set_arg_buffer(idn, 0, prev.weights));
      NN(nn_set_arg_int(idn, 1, prev.neurons + 1));
      updates_.push_back({l,
                          {ida, 2, {(unsigned)cur.neurons, (unsigned)(prev.neurons + 1)}, {0, 0}, false},
                          {idn, 1, {(unsigned)cur.neurons, 0}, {0, 0}, false}});
    }
  }

  std::vector<Layer> layers_;
  int target_ = -1, next_id_ = 0;
  std::vector<Exec> forward_, backward_;
  std::vector<Upd> updates_;
};

struct NetSpec {
  std::vector<int> sizes, acts;
};

// D/net.txt, read before the library is initialised so that a bad file costs no device work.
NetSpec read_spec(const std::string &dir) {
  std::ifstream spec(dir + "/net.txt");
  if (!spec) die("cannot open " + dir + "/net.txt");
  std::string l1, l2;
  std::getline(spec, l1);
  std::getline(spec, l2);
  NetSpec ns{parse_ints(l1), parse_ints(l2)};
  if (ns.sizes.size() < 2 || ns.sizes.size() != ns.acts.size())
    die(dir + "/net.txt: need at least two layer sizes and one activation per layer");
  for (int n : ns.sizes)
    if (n <= 0) die(dir + "/net.txt: layer sizes must be positive");
  return ns;
}

int run_files(const std::string &dir, const NetSpec &ns, int steps) {
  const std::vector<int> &sizes = ns.sizes, &acts = ns.acts;
  DenseNet net(sizes, acts);
  for (size_t l = 0; l + 1 < net.size(); ++l)
    net.set_weights(l, read_f32(dir + "/w" + std::to_string(l) + ".f32", (size_t)net.weight_count(l)));
  const int n_in = sizes.front(), n_out = sizes.back();
  const std::vector<float> x = read_f32(dir + "/x.f32", (size_t)steps * n_in);
  const std::vector<float> t = read_f32(dir + "/t.f32", (size_t)steps * n_out);
  std::vector<float> y((size_t)steps * n_out);
  for (int s = 0; s < steps; ++s)
    net.step(x.data() + (size_t)s * n_in, t.data() + (size_t)s * n_out, y.data() + (size_t)s * n_out);
  NN(nn_finish(60000));
  write_f32(dir + "/y.f32", y);
  for (size_t l = 0; l + 1 < net.size(); ++l) {
    const Layer &L = net.layer(l);
    const long long n = net.weight_count(l);
    write_f32(dir + "/w" + std::to_string(l) + ".out.f32", net.read(L.weights, n));
    write_f32(dir + "/m" + std::to_string(l) + ".out.f32", net.read(L.m, n));
    write_f32(dir + "/v" + std::to_string(l) + ".out.f32", net.read(L.v, n));
  }
  std::printf("{\"harness\": \"dense_online\", \"steps\": %d, \"layers\": %zu}\n", steps, net.size());
  return 0;
}

int run_synthetic(int steps) {
  const std::vector<int> sizes = {240, 500, 500, 3};
  const std::vector<int> acts = {NN_ACT_NONE, NN_ACT_TANH, NN_ACT_SIGMOID, NN_ACT_NONE};
  DenseNet net(sizes, acts);
  Rng rng(42);
  for (size_t l = 0; l + 1 < net.size(); ++l) {
    const double k = 1.0 / std::sqrt((double)sizes[l]);
    std::vector<float> w((size_t)net.weight_count(l));
    for (float &v : w) v = rng.range(-k, k);
    net.set_weights(l, w);
  }
  const int pool = 1000, n_in = sizes.front(), n_out = sizes.back();
  std::vector<float> x((size_t)pool * n_in), t((size_t)pool * n_out), y((size_t)n_out);
  for (float &v : x) v = rng.range(-1.0, 1.0);
  for (float &v : t) v = rng.range(0.0, 1.0);
  for (int s = 0; s < 3; ++s) net.step(x.data(), t.data(), y.data());  // warm-up
  NN(nn_finish(60000));
  double mse = 0.0;
  const auto t0 = std::chrono::steady_clock::now();
  for (int s = 0; s < steps; ++s) {
    const int i = s % pool;
    net.step(x.data() + (size_t)i * n_in, t.data() + (size_t)i * n_out, y.data());
    mse = 0.0;
    for (int j = 0; j < n_out; ++j) {
      const double d = (double)y[j] - t[(size_t)i * n_out + j];
      mse += d * d / n_out;
    }
  }
  NN(nn_finish(60000));
  const double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  std::printf("{\"harness\": \"dense_online\", \"steps\": %d, \"seconds\": %.6f, \"steps_per_s\": %.1f, "
              "\"last_mse\": %.6g}\n",
              steps, sec, steps / sec, mse);
  return 0;
}

}  // namespace

int main(int argc, char **argv) {
  std::string dir;
  int steps = 0, device = 0;
  bool synthetic = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--dir" && i + 1 < argc) dir = argv[++i];
    else if (a == "--steps" && i + 1 < argc) steps = std::atoi(argv[++i]);
    else if (a == "--device" && i + 1 < argc) device = std::atoi(argv[++i]);
    else if (a == "--synthetic") synthetic = true;
    else die("unknown argument " + a + " (usage: --dir D --steps N | --synthetic --steps N; [--device K])");
  }
  if (steps <= 0 || (dir.empty() && !synthetic)) die("usage: --dir D --steps N | --synthetic --steps N; [--device K]");
  NetSpec ns;
  if (!synthetic) ns = read_spec(dir);
  NN(nn_init(device, 0));
  const int rc = synthetic ? run_synthetic(steps) : run_files(dir, ns, steps);
  NN(nn_shutdown());
  return rc;
}
