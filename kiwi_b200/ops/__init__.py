"""kiwi_b200.ops"""
