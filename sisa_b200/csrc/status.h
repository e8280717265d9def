// Status bits and return codes shared by device and host code (defined in the public C header).
#pragma once
#include "sisa_b200.h"
