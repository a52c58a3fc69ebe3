#pragma once

#include <nrn/connectivity/connect.h>
#include <nrn/connectivity/connectivity_tensor.h>
#include <nrn/connectivity/options.h>
#include <nrn/connectivity/topology/distance_dependent.h>
#include <nrn/connectivity/topology/random.h>
#include <nrn/connectivity/topology/topology.h>
