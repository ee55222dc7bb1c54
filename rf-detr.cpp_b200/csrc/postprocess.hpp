// Detection result ownership: arrays and masks are malloc'd blocks released by
// rfdetr_detections_free (declared in rfdetr.h).
#pragma once

#include "rfdetr.h"
