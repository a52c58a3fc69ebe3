#pragma once

#include <nrn/synapse/ampa.h>
#include <nrn/synapse/double_exponential.h>
#include <nrn/synapse/exponential.h>
#include <nrn/synapse/options.h>
#include <nrn/synapse/static.h>
