"""Files that plug this package into other frameworks."""
