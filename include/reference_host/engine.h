// engine.h for a reference host (the reference's src/main.cpp) built on vela_b200: place this directory ahead of the
// reference's src/ on the include path and the host's `#include "engine.h"` gets vela_b200's DevModel / Engine /
// EngineConfig instead of the reference's engine.  Everything else the host includes stays its own.
#pragma once
#include "common.h"     // the host's CUDA runtime include and helpers, which its own engine.h brought in
#include "poisd.h"      // meow::Poisd: DevModel::load takes the host's parsed model
#include "vela_b200_engine.hpp"
