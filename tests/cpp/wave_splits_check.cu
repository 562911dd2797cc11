// Host-only check of the split-K rule of the weight-gradient and LSTM products (wave_splits in
// nn_in_trading_b200/csrc/wgrad.cuh): reads "tiles cap" pairs on stdin and prints
// "tiles cap splits" for each.  No device code runs.
#include <cstdio>

#include "../../include/nn_b200.h"
#include "../../nn_in_trading_b200/csrc/wgrad.cuh"

int main() {
  long long tiles = 0, cap = 0;
  while (std::scanf("%lld %lld", &tiles, &cap) == 2) std::printf("%lld %lld %d\n", tiles, cap, nn::wave_splits(tiles, cap));
  return 0;
}
