// The reference's Objective-C bridge (include/objc.h) is not needed on the
// B200 backend: CUDA is a C API.  Kept so that code including <objc.h> builds.
#pragma once
