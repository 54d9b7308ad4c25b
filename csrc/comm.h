#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
