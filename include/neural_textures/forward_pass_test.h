// neural_textures/forward_pass_test.h -- replaces tests/forward_pass_test.h:6 of
// mavenkim2/neural_textures with the same declaration.  Returns true when the 12 -> 16 -> 16
// known-answer test passes on the current CUDA device (prints the first mismatch otherwise).
#pragma once

namespace neural_textures {

#if defined(__GNUC__)
__attribute__((visibility("default")))
#endif
bool RunForwardPassTest();

}  // namespace neural_textures
