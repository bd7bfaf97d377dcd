"""einjax_b200 package (placeholder)."""
