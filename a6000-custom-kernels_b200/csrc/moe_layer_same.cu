// moe_layer_same.cu -- fused layer kernels for the remaining types, with the
// down tensor of the gate/up type.
#include "moe_layer_launch.cuh"
namespace moe {
template cudaError_t launch_layer_t<T_Q4_0, T_Q4_0>(const LayerArgs &, int, size_t, cudaStream_t);
template cudaError_t launch_layer_t<T_Q5_0, T_Q5_0>(const LayerArgs &, int, size_t, cudaStream_t);
template cudaError_t launch_layer_t<T_Q8_0, T_Q8_0>(const LayerArgs &, int, size_t, cudaStream_t);
template cudaError_t launch_layer_t<T_Q5_K, T_Q5_K>(const LayerArgs &, int, size_t, cudaStream_t);
template cudaError_t launch_layer2_t<T_Q4_0, T_Q4_0>(const Layer2Args &, int, size_t, cudaStream_t);
template cudaError_t launch_layer2_t<T_Q5_0, T_Q5_0>(const Layer2Args &, int, size_t, cudaStream_t);
template cudaError_t launch_layer2_t<T_Q8_0, T_Q8_0>(const Layer2Args &, int, size_t, cudaStream_t);
template cudaError_t launch_layer2_t<T_Q5_K, T_Q5_K>(const Layer2Args &, int, size_t, cudaStream_t);
}  // namespace moe
