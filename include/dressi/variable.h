// Forwards to the C++ graph API of libdressi_b200 (dressi/dressi.h), so a
// program that includes the reference's dressi/variable.h builds unchanged.
#pragma once
#include "dressi.h"
