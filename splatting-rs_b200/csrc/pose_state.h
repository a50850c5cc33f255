// The host pose refinement's state (sp_pose_refinement), shared by pose.cpp and the device
// copy in pose_device.cu: the initial cameras, one ViewState per view, the SharedState.
#pragma once

#include <vector>

#include "pose_math.h"

struct sp_pose_refinement {
    std::vector<sp_pinhole_camera> initial;
    std::vector<splat::pose::ViewState> views;
    splat::pose::SharedState shared{};
};
