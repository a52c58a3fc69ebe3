// nrn.h -- umbrella header of the nrn:: API (same role as the reference's include/nrn.h).
#pragma once

#include <nrn/nrn.h>
