"""Emission (skeleton + parameters -> text) and the shape -> kernel dispatch registry."""
