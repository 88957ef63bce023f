// TEST INFRASTRUCTURE ONLY (oracle). Stand-in for the reference's include/breeze/generation.h when
// its src/text_split.cpp is compiled on its own: the reference header pulls in the ggml-based
// model headers, while text_split.cpp needs only the two declarations of its own functions
// (sharjeel103/bz-ggml include/breeze/generation.h:40-45).
#pragma once

#include <string>
#include <vector>

namespace breeze {
std::vector<std::string> split_text(const std::string & text, int budget, int first_budget = 0);
double estimate_seconds(const std::string & text);
}
