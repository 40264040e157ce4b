"""Calibration records (tempo/calib/2): measured rates that replace a plugin's MODEL or
NOT_MEASURED rates."""
