"""kiwi_b200.utils"""
