"""Plugins behind the ``tempo/arch/1`` contract: ``sm100`` (B200, the product) and small
falsifier plugins used by the boundary gates."""
