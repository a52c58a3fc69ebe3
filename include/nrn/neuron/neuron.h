#pragma once

#include <nrn/neuron/adex.h>
#include <nrn/neuron/izhikevich.h>
#include <nrn/neuron/lif.h>
#include <nrn/neuron/options.h>
