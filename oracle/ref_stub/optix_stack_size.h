#pragma once
#include "optix_host.h"
