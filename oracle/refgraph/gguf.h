// Stand-in (test infrastructure; see ggml.h). The reference's reader
// (src/gguf_load.cpp) parses GGUF itself and needs nothing from here.
#pragma once
#include "ggml.h"
