"""Lower-bound period model and wave arithmetic."""
