"""CPU oracle for sqrt-block attention: test infrastructure, never a product path."""
