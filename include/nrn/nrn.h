// nrn/nrn.h -- everything of the nrn:: API.
#pragma once

#include <nrn/config/config.h>
#include <nrn/connectivity/connectivity.h>
#include <nrn/core/device.h>
#include <nrn/core/module.h>
#include <nrn/core/options.h>
#include <nrn/core/state.h>
#include <nrn/core/types.h>
#include <nrn/monitor/monitor.h>
#include <nrn/network/network.h>
#include <nrn/neuron/neuron.h>
#include <nrn/plasticity/plasticity.h>
#include <nrn/simulation/simulation.h>
#include <nrn/synapse/synapse.h>

using namespace nrn::literals;
