"""mdl_b200 package."""
