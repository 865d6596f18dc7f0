// moe_layer_q4k.cu -- fused layer kernels with Q4_K gate/up.
#include "moe_layer_launch.cuh"
namespace moe {
template cudaError_t launch_layer_t<T_Q4_K, T_Q2_K>(const LayerArgs &, int, size_t, cudaStream_t);
template cudaError_t launch_layer_t<T_Q4_K, T_Q3_K>(const LayerArgs &, int, size_t, cudaStream_t);
template cudaError_t launch_layer_t<T_Q4_K, T_Q4_K>(const LayerArgs &, int, size_t, cudaStream_t);
template cudaError_t launch_layer_t<T_Q4_K, T_Q6_K>(const LayerArgs &, int, size_t, cudaStream_t);
template cudaError_t launch_layer2_t<T_Q4_K, T_Q2_K>(const Layer2Args &, int, size_t, cudaStream_t);
template cudaError_t launch_layer2_t<T_Q4_K, T_Q3_K>(const Layer2Args &, int, size_t, cudaStream_t);
template cudaError_t launch_layer2_t<T_Q4_K, T_Q4_K>(const Layer2Args &, int, size_t, cudaStream_t);
template cudaError_t launch_layer2_t<T_Q4_K, T_Q6_K>(const Layer2Args &, int, size_t, cudaStream_t);
}  // namespace moe
