// Stand-in (test infrastructure; see ggml.h).
#pragma once
#include "ggml-backend.h"
