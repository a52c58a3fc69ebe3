#pragma once

#include <nrn/monitor/recorder.h>
#include <nrn/monitor/spike_recorder.h>
#include <nrn/monitor/state_recorder.h>
