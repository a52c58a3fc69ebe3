#pragma once

#include <nrn/plasticity/options.h>
#include <nrn/plasticity/plasticity_rule.h>
#include <nrn/plasticity/stdp.h>
