#pragma once

#include <nrn/network/population.h>
#include <nrn/network/region.h>
