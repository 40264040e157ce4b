"""The atom IR (channel footprints) and its serialisation."""
