"""Drop-in replacements for the reference's ``runtime`` modules on the gate/up path."""
