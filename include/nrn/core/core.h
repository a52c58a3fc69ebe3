#pragma once

#include <nrn/core/device.h>
#include <nrn/core/module.h>
#include <nrn/core/options.h>
#include <nrn/core/state.h>
