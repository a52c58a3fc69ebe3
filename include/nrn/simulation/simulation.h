#pragma once

#include <nrn/simulation/clock.h>
#include <nrn/simulation/options.h>
#include <nrn/simulation/runner.h>
#include <nrn/simulation/spike_buffer.h>
